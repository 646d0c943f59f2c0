"""``LearnedAddressSparseAttention`` on the sm_100a kernels.

Drop-in for the reference module of the same name
(``routing_attention/models/attention.py:409-501``) and its address module
(``routing_attention/models/learned_address.py:12-56``): same constructor
signature, same submodule names (``q_proj``, ``k_proj``, ``v_proj``,
``out_proj``, ``address.q_addr_proj``, ``address.k_addr_proj``), so reference
``state_dict``s load unchanged.  Projections, address normalisation and
``out_proj`` stay in PyTorch; retrieval + sparse attention run in the CUDA
library.

Differences from the reference module, all deliberate:
  * no ``RoutingRetriever`` is built, so no ``max_seq_len**2`` causal mask is
    allocated (``retrieval/index.py:112-113``);
  * both module paths call the same exact kernel.  With
    ``use_fused_sparse=False`` the addresses are first rounded to
    ``retrieval_config.dtype`` (fp16 by default), reproducing the non-fused
    path's retrieval numerics (``retrieval/index.py:188-207``);
  * the fused path is forward-only like the reference's (``@torch.no_grad``,
    ``kernels/fused_sparse.py:327``); the non-fused path trains: its sparse
    attention has a CUDA backward for q, k and v and applies the module's
    attention-probability dropout in training mode (its own counter-based
    generator, so the masks differ from PyTorch's nn.Dropout draws).
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Literal, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .causal_topk import causal_topk
from .fused_sparse import fused_sparse_attention, sparse_meat_attention


@dataclass
class RetrievalConfig:
    """Fields of ``routing_attention/retrieval/index.py:82-98``; only
    ``top_k``, ``use_fused_sparse`` and ``dtype`` influence this build."""

    method: str = "auto"
    top_k: int = 32
    max_seq_len: int = 8192
    oversample: int = 4
    dtype: Literal["float32", "float16", "bfloat16"] = "float16"
    brute_force_max_seq: int = 2048
    faiss_flat_max_seq: int = 16384
    hnsw_m: int = 32
    hnsw_ef_search: int = 64
    use_gpu: bool = True
    apply_to_key_vector: bool = False
    use_fused_sparse: bool = False


def retrieval_config_from_dict(d: dict | None) -> RetrievalConfig:
    """Like ``retrieval/index.py:372-387``: unknown keys are ignored."""
    d = d or {}
    names = {f.name for f in fields(RetrievalConfig)}
    return RetrievalConfig(**{k: v for k, v in d.items() if k in names})


def _resolve_retrieval_cfg(cfg: RetrievalConfig | dict | None, top_k: int) -> RetrievalConfig:
    if isinstance(cfg, dict):
        return retrieval_config_from_dict(cfg)
    return cfg or RetrievalConfig(top_k=top_k)


class LearnedAddressModule(nn.Module):
    """Query/key address projections + L2 normalisation (``learned_address.py:12-56``)."""

    def __init__(
        self,
        d_model: int,
        address_dim: int = 32,
        similarity: Literal["symmetric", "asymmetric"] = "asymmetric",
        normalize: bool = True,
    ):
        super().__init__()
        self.d_model = d_model
        self.address_dim = address_dim
        self.similarity = similarity
        self.normalize = normalize
        self.q_addr_proj = nn.Linear(d_model, address_dim)
        self.k_addr_proj = nn.Linear(d_model, address_dim) if similarity == "asymmetric" else None
        # inference on CUDA: both projections + normalisation in one kernel (wf_address_projection)
        self.fused_projection = True

    def forward_query_key(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        if self._use_fused_projection(hidden):
            return self._fused_query_key(hidden)
        q = self.q_addr_proj(hidden)
        k = self.k_addr_proj(hidden) if self.k_addr_proj is not None else q
        if self.normalize:
            q = F.normalize(q, dim=-1)
            k = F.normalize(k, dim=-1)
        return q, k

    def _use_fused_projection(self, hidden: torch.Tensor) -> bool:
        """One fused kernel (``wf_address_projection``) when no gradient is needed."""
        if not (self.fused_projection and hidden.is_cuda) or hidden.dtype not in _DTYPES.values():
            return False
        return not (torch.is_grad_enabled() and (hidden.requires_grad or any(p.requires_grad for p in self.parameters())))

    def _fused_query_key(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        from .address_projection import StackedAddressWeights, address_projection

        if not hasattr(self, "_stacked"):
            self._stacked = StackedAddressWeights()
        layers = [self.q_addr_proj] + ([self.k_addr_proj] if self.k_addr_proj is not None else [])
        w, b = self._stacked.get(layers)
        out = address_projection(hidden, w, b, self.address_dim, normalize=self.normalize)
        q = out[..., : self.address_dim]
        k = out[..., self.address_dim:] if self.k_addr_proj is not None else q
        return q, k

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        q, _ = self.forward_query_key(hidden)
        return q

    def retrieval_scores(self, hidden: torch.Tensor) -> torch.Tensor:
        q, k = self.forward_query_key(hidden)
        return torch.matmul(q, k.transpose(-2, -1))


_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


class LearnedAddressSparseAttention(nn.Module):
    """Learned addresses pick K causal candidates; softmax attention runs on that subset."""

    def __init__(
        self,
        d_model: int,
        n_heads: int,
        top_k: int = 32,
        address_dim: int = 32,
        similarity: Literal["symmetric", "asymmetric"] = "asymmetric",
        dropout: float = 0.1,
        address_module: LearnedAddressModule | None = None,
        retrieval_config: RetrievalConfig | dict | None = None,
        pad_mode: str = "reference",
        mask_padded_keys: bool = False,
    ):
        super().__init__()
        assert d_model % n_heads == 0
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.scale = self.head_dim ** -0.5
        self.top_k = top_k
        self.pad_mode = pad_mode
        # Honour attn_mask (B, T) as a key-padding mask on the fused path; the
        # reference ignores it there, so the default keeps its behaviour.
        self.mask_padded_keys = mask_padded_keys
        self._retrieval_cfg = _resolve_retrieval_cfg(retrieval_config, top_k)
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.dropout = nn.Dropout(dropout)
        self.address = address_module or LearnedAddressModule(
            d_model=d_model, address_dim=address_dim, similarity=similarity
        )

    def set_address_module(self, address_module: LearnedAddressModule) -> None:
        self.address = address_module

    def forward(
        self,
        x: torch.Tensor,
        attn_mask: Optional[torch.Tensor] = None,
        return_attention: bool = False,
        **kwargs,
    ):
        # attn_mask is ignored, as on the reference's sparse path (attention.py:456-490), unless the
        # module was built with mask_padded_keys=True (fused path: padded keys are never retrieved).
        B, T, D = x.shape
        q = self.q_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        q_addr, k_addr = self.address.forward_query_key(x)
        if self._retrieval_cfg.use_fused_sparse:
            key_mask = attn_mask if (self.mask_padded_keys and attn_mask is not None and not bool(attn_mask.all())) else None
            meat, candidate_idx = fused_sparse_attention(
                q_addr, k_addr, q, k, v, self.top_k, self.scale, pad_mode=self.pad_mode, key_mask=key_mask
            )
        else:
            rdt = _DTYPES.get(self._retrieval_cfg.dtype, torch.float16)
            candidate_idx = causal_topk(q_addr.to(rdt), k_addr.to(rdt), self.top_k, pad_mode=self.pad_mode)
            meat = sparse_meat_attention(
                q, k, v, candidate_idx, self.scale, mask_negative=self.pad_mode == "masked",
                dropout_p=self.dropout.p if self.training else 0.0,
            )
        out = meat.transpose(1, 2).contiguous().view(B, T, D)
        out = self.out_proj(out)
        if return_attention:
            # Same debug map as attention.py:492-500 (1/K at each retrieved position), built vectorised.
            k_eff = candidate_idx.shape[-1]
            attn_dense = torch.zeros(B, T, T, device=x.device)
            if k_eff > 0:
                idx = candidate_idx.long()
                # masked pad slots (-1) are redirected to slot 0, which always holds a real key
                idx = torch.where(idx >= 0, idx, idx[..., :1])
                attn_dense.scatter_(2, idx, 1.0 / k_eff)
            return out, attn_dense
        return out


class KeyVectorSparseAttention(nn.Module):
    """Key-vector retrieval baseline (``routing_attention/models/attention.py:296-406``).

    The search vectors are head means of the Q/K projections (R = head_dim) and the
    same fused retrieval + sparse attention kernels run on them.  The reference's
    ``_search_vectors(k, q)`` is called as ``_search_vectors(q, k)`` on both of its
    paths (``attention.py:341-343, 349, 384``), so its *query* search vector is the
    head mean of the keys and its *key* search vector the head mean of the queries;
    this module reproduces that.  ``apply_to_key_vector=True`` rounds the search
    vectors to ``retrieval_config.dtype`` first (the ``RoutingRetriever`` numerics).
    Rows i < K-1 get the reference pads of ``_finalize_causal_topk`` on every path
    (the reference's inline path leaves arbitrary masked indices there).
    """

    def __init__(
        self,
        d_model: int,
        n_heads: int,
        top_k: int = 32,
        dropout: float = 0.1,
        retrieval_config: RetrievalConfig | dict | None = None,
        pad_mode: str = "reference",
    ):
        super().__init__()
        assert d_model % n_heads == 0
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.scale = self.head_dim ** -0.5
        self.top_k = top_k
        self.pad_mode = pad_mode
        self._retrieval_cfg = _resolve_retrieval_cfg(retrieval_config, top_k)
        self.use_fast_retrieval = self._retrieval_cfg.apply_to_key_vector
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.dropout = nn.Dropout(dropout)

    def _search_vectors(self, q: torch.Tensor, k: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(query search, key search) as the reference computes them: (mean_h k, mean_h q)."""
        return k.mean(dim=1).contiguous(), q.mean(dim=1).contiguous()

    def forward(self, x: torch.Tensor, attn_mask: Optional[torch.Tensor] = None, return_attention: bool = False,
                **kwargs):
        B, T, D = x.shape
        q = self.q_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        qs, ks = self._search_vectors(q, k)
        if self._retrieval_cfg.use_fused_sparse:
            meat, candidate_idx = fused_sparse_attention(qs, ks, q, k, v, self.top_k, self.scale,
                                                         pad_mode=self.pad_mode)
        else:
            if self.use_fast_retrieval:
                rdt = _DTYPES.get(self._retrieval_cfg.dtype, torch.float16)
                qs, ks = qs.to(rdt), ks.to(rdt)
            candidate_idx = causal_topk(qs, ks, self.top_k, pad_mode=self.pad_mode)
            meat = sparse_meat_attention(q, k, v, candidate_idx, self.scale,
                                         mask_negative=self.pad_mode == "masked",
                                         dropout_p=self.dropout.p if self.training else 0.0)
        out = self.out_proj(meat.transpose(1, 2).contiguous().view(B, T, D))
        if return_attention:
            k_eff = candidate_idx.shape[-1]
            attn_dense = torch.zeros(B, T, T, device=x.device)
            if k_eff > 0:
                idx = candidate_idx.long()
                idx = torch.where(idx >= 0, idx, idx[..., :1])
                attn_dense.scatter_(2, idx, 1.0 / k_eff)
            return out, attn_dense
        return out


class RoutingSparseAttention(nn.Module):
    """Router-driven sparse attention (``routing_attention/models/attention.py:504-617``).

    The router's (B, T, R) routing vectors are the search vectors of the same fused
    retrieval + sparse-attention kernels: ``RouterMLP.forward_query_key`` (or
    ``PerLayerRouter`` for ``layer_idx``, or the concatenated local + global vectors
    of a ``MultiScaleRouter``, R = 2 * routing_dim).  Same constructor, submodule
    names (``router``, ``q_proj``, ``k_proj``, ``v_proj``, ``out_proj``,
    ``_key_baseline``) and ``forward`` contract as the reference.  The non-fused
    path rounds the routing vectors to ``retrieval_config.dtype`` before retrieval
    (the ``RoutingRetriever`` numerics), except with a ``MultiScaleRouter``, whose
    ``retrieve_indices`` merges the two routers' candidates as the reference does.
    Per-head routing vectors (B, T, H, R) are rejected with ``ValueError`` on the
    fused path, as the reference operator rejects non-3-D search vectors.
    """

    def __init__(
        self,
        d_model: int,
        n_heads: int,
        router: nn.Module,
        top_k: int = 32,
        dropout: float = 0.1,
        layer_idx: int = 0,
        retrieval_mode: Literal["routing", "key_vector"] = "routing",
        retrieval_config: RetrievalConfig | dict | None = None,
        pad_mode: str = "reference",
    ):
        super().__init__()
        assert d_model % n_heads == 0
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.scale = self.head_dim ** -0.5
        self.top_k = top_k
        self.router = router
        self.layer_idx = layer_idx
        self.retrieval_mode = retrieval_mode
        self.pad_mode = pad_mode
        self._retrieval_cfg = _resolve_retrieval_cfg(retrieval_config, top_k)
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.dropout = nn.Dropout(dropout)
        if retrieval_mode == "key_vector":
            self._key_baseline = KeyVectorSparseAttention(d_model, n_heads, top_k, dropout,
                                                          retrieval_config=retrieval_config, pad_mode=pad_mode)

    def _get_query_key_routing(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        from .router import PerLayerRouter

        if isinstance(self.router, PerLayerRouter):
            return self.router.forward_query_key(x, self.layer_idx)
        if hasattr(self.router, "forward_query_key"):
            return self.router.forward_query_key(x)
        r = self.router(x)
        return r, r

    def forward(self, x: torch.Tensor, attn_mask: Optional[torch.Tensor] = None, return_attention: bool = False,
                precomputed_routing: Optional[torch.Tensor] = None):
        from .router import MultiScaleRouter

        if self.retrieval_mode == "key_vector":
            return self._key_baseline(x, attn_mask=attn_mask, return_attention=return_attention)
        B, T, D = x.shape
        q = self.q_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        if self._retrieval_cfg.use_fused_sparse:
            q_r, k_r = self._get_query_key_routing(x)
            meat, candidate_idx = fused_sparse_attention(q_r, k_r, q, k, v, self.top_k, self.scale,
                                                         pad_mode=self.pad_mode)
        else:
            if isinstance(self.router, MultiScaleRouter):
                candidate_idx = self.router.retrieve_indices(x, self.top_k, self.layer_idx).to(torch.int32)
            else:
                q_r, k_r = self._get_query_key_routing(x)
                rdt = _DTYPES.get(self._retrieval_cfg.dtype, torch.float16)
                candidate_idx = causal_topk(q_r.to(rdt), k_r.to(rdt), self.top_k, pad_mode=self.pad_mode)
            meat = sparse_meat_attention(q, k, v, candidate_idx, self.scale, mask_negative=self.pad_mode == "masked",
                                         dropout_p=self.dropout.p if self.training else 0.0)
        out = self.out_proj(meat.transpose(1, 2).contiguous().view(B, T, D))
        if return_attention:
            k_eff = candidate_idx.shape[-1]
            attn_dense = torch.zeros(B, T, T, device=x.device)
            if k_eff > 0:
                idx = candidate_idx.long()
                idx = torch.where(idx >= 0, idx, idx[..., :1])
                attn_dense.scatter_(2, idx, 1.0 / k_eff)
            return out, attn_dense
        return out
