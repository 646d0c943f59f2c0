"""Wayfinder causal learned-address retrieval + sparse attention on B200 (sm_100a).

Public API (names and arguments of the reference's ``routing_attention``):
  causal_topk, fused_sparse_attention, sparse_meat_attention, SparseMeatConfig,
  LearnedAddressSparseAttention, LearnedAddressModule, RetrievalConfig,
  TransformerLM (the decoder harness); HostFusedSparseAttention runs the fused
  op on pinned host tensors with upload, compute and download overlapped.

The compute runs in ``libwayfinder_sm100.so`` (C ABI: ``include/wayfinder.h``);
there is no CPU path.  Kernel faults that do not stop a kernel (an out-of-range
index, a bounded wait that timed out) raise ``RuntimeError`` at the next call on
the device, or at ``check_status()``, which waits for the device's queued work.
"""

from ._lib import check_status, load_library
from .attention import (
    KeyVectorSparseAttention,
    LearnedAddressModule,
    LearnedAddressSparseAttention,
    RetrievalConfig,
    RoutingSparseAttention,
    retrieval_config_from_dict,
)
from .router import MultiScaleRouter, PerLayerRouter, RouterMLP
from .causal_topk import causal_topk, causal_topk_available, promote_compute_dtype
from .decoder import DenseSDPAAttention, TransformerBlock, TransformerLM
from .graphs import CapturedForward
from .host_pipeline import HostFusedSparseAttention, host_fused_sparse_attention
from .fused_sparse import (
    SparseMeatConfig,
    fused_sparse_attention,
    fused_sparse_attention_available,
    sparse_meat_attention,
)

__all__ = [
    "load_library",
    "check_status",
    "causal_topk",
    "causal_topk_available",
    "promote_compute_dtype",
    "fused_sparse_attention",
    "fused_sparse_attention_available",
    "sparse_meat_attention",
    "HostFusedSparseAttention",
    "CapturedForward",
    "host_fused_sparse_attention",
    "SparseMeatConfig",
    "LearnedAddressModule",
    "LearnedAddressSparseAttention",
    "KeyVectorSparseAttention",
    "RoutingSparseAttention",
    "RouterMLP",
    "PerLayerRouter",
    "MultiScaleRouter",
    "RetrievalConfig",
    "retrieval_config_from_dict",
    "DenseSDPAAttention",
    "TransformerBlock",
    "TransformerLM",
]
