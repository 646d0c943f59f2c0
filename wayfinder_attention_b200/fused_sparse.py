"""Sparse softmax attention over retrieved rows, and the fused retrieval + attention op.

Drop-in for ``routing_attention.kernels.fused_sparse`` of the reference:
  * ``sparse_meat_attention``  <- ``fused_sparse.py:275-324``
  * ``fused_sparse_attention`` <- ``fused_sparse.py:327-356``
  * ``SparseMeatConfig``       <- ``fused_sparse.py:30-38`` (accepted, ignored)

The arithmetic is that of ``sparse_meat_attention_reference``
(``fused_sparse.py:80-94``): gather K/V rows at indices shared by all heads,
scaled dot products, softmax over the K retrieved rows, weighted sum of V,
evaluated in fp32 and rounded once to the output dtype (the reference's
``batched`` GPU path runs its softmax in the input dtype instead).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .causal_topk import _launch_topk, pad_mode_code, promote_compute_dtype


@dataclass
class SparseMeatConfig:
    """Launch tuning of the reference (``fused_sparse.py:30-38``); the CUDA kernel ignores it."""

    method: str = "auto"
    block_d: int | None = None
    k_pad: int | None = None
    num_warps: int = 4
    compute_dtype: str | None = None


def _attn_operand(t: torch.Tensor) -> torch.Tensor:
    """Return ``t`` if the kernel can read it in place (unit last stride, 16-byte rows), else a compact copy."""
    esz = t.element_size()
    ok = (
        t.stride(-1) == 1
        and t.data_ptr() % 16 == 0
        and all((s * esz) % 16 == 0 for s in t.stride()[:-1])
    )
    return t if ok else t.contiguous()


def _check_meat_shapes(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError(f"expected (B,H,T,D) q/k/v, got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if k.shape != v.shape:
        raise ValueError(f"k/v shape mismatch: {tuple(k.shape)} vs {tuple(v.shape)}")
    if q.shape[0] != k.shape[0] or q.shape[1] != k.shape[1] or q.shape[3] != k.shape[3]:
        raise ValueError(f"q/k shape mismatch: {tuple(q.shape)} vs {tuple(k.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError(f"q/k/v dtype mismatch: {q.dtype}, {k.dtype}, {v.dtype}")


def _launch_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    indices: torch.Tensor,
    scale: float,
    *,
    mask_negative: bool,
    out_dtype: torch.dtype | None,
    status: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    drop_rate: float = 0.0,
    drop_seed: int = 0,
) -> torch.Tensor:
    dev = _lib.require_cuda(q, k, v, indices)
    lib = _lib.load_library()
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    K = indices.shape[-1]
    if indices.dim() != 3 or indices.shape[0] != B or indices.shape[1] != Tq:
        raise ValueError(f"indices must have shape {(B, Tq, K)}, got {tuple(indices.shape)}")
    if out is None:
        out = torch.empty(B, H, Tq, D, dtype=out_dtype or q.dtype, device=dev)
    elif tuple(out.shape) != (B, H, Tq, D) or out.device != dev or (out_dtype and out.dtype != out_dtype):
        raise ValueError(f"out must be a {(B, H, Tq, D)} tensor on {dev}")
    if K == 0:
        # softmax over an empty set: the reference's sum over zero rows is 0
        return out.zero_()
    q, k, v = _attn_operand(q), _attn_operand(k), _attn_operand(v)
    flags = _lib.WF_ATTN_MASK_NEGATIVE if mask_negative else 0
    st = _lib.status_arg(dev, status)
    with torch.cuda.device(dev):
        if drop_rate > 0.0:
            rc = lib.wf_sparse_attention_dropout(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q.dtype), indices.data_ptr(),
                B, H, Tq, Tk, D, K, _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(indices),
                float(scale), flags, float(drop_rate), int(drop_seed), out.data_ptr(), _lib.dtype_code(out.dtype),
                _lib.strides(out), st, _lib.stream_ptr(dev),
            )
        else:
            rc = lib.wf_sparse_attention(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q.dtype), indices.data_ptr(),
                B, H, Tq, Tk, D, K,
                _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(indices),
                float(scale), flags, out.data_ptr(), _lib.dtype_code(out.dtype), _lib.strides(out),
                st, _lib.stream_ptr(dev),
            )
    _lib.check(rc)
    _lib.status_after(dev, status)
    return out


def _launch_attention_backward(q, k, v, indices, dout, scale, mask_negative, status=None, drop_rate=0.0,
                               drop_seed=0):
    """(dq, dk, dv) of the sparse attention via ``wf_sparse_attention_backward``."""
    dev = _lib.require_cuda(q, k, v, indices, dout)
    lib = _lib.load_library()
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    K = indices.shape[-1]
    q, k, v = _attn_operand(q), _attn_operand(k), _attn_operand(v)
    dout = _attn_operand(dout.to(q.dtype))
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    n = lib.wf_sparse_attention_backward_workspace_bytes(B, H, Tq, Tk, K)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=dev)
    st = _lib.status_arg(dev, status)
    with torch.cuda.device(dev):
        rc = lib.wf_sparse_attention_backward(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q.dtype), indices.data_ptr(),
            B, H, Tq, Tk, D, K, _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(indices),
            dout.data_ptr(), _lib.strides(dout), float(scale), _lib.WF_ATTN_MASK_NEGATIVE if mask_negative else 0,
            float(drop_rate), int(drop_seed), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), _lib.dtype_code(q.dtype), _lib.strides(dq),
            _lib.strides(dk), _lib.strides(dv), ws.data_ptr(), ws.numel(),
            st, _lib.stream_ptr(dev),
        )
    _lib.check(rc)
    _lib.status_after(dev, status)
    return dq, dk, dv


class _SparseMeatFunction(torch.autograd.Function):
    """Sparse attention with a backward (``wf_sparse_attention_backward``); indices get no gradient."""

    @staticmethod
    def forward(ctx, q, k, v, indices, scale, mask_negative, out_dtype, drop_rate, drop_seed):
        out = _launch_attention(q, k, v, indices, scale, mask_negative=mask_negative, out_dtype=out_dtype,
                                drop_rate=drop_rate, drop_seed=drop_seed)
        ctx.save_for_backward(q, k, v, indices)
        ctx.scale = scale
        ctx.mask_negative = mask_negative
        ctx.drop = (drop_rate, drop_seed)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, indices = ctx.saved_tensors
        dq, dk, dv = _launch_attention_backward(q, k, v, indices, dout, ctx.scale, ctx.mask_negative,
                                                drop_rate=ctx.drop[0], drop_seed=ctx.drop[1])
        return dq, dk, dv, None, None, None, None, None, None


def sparse_meat_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    indices: torch.Tensor,
    scale: float,
    *,
    method: str = "auto",
    config: SparseMeatConfig | None = None,
    out_dtype: torch.dtype | None = None,
    mask_negative: bool = False,
    status: torch.Tensor | None = None,
    dropout_p: float = 0.0,
    dropout_seed: int | None = None,
) -> torch.Tensor:
    """Multi-head sparse attention on pre-selected indices shared across heads.

    q: (B, H, T, D); k, v: (B, H, Tk, D); indices: (B, T, K) (cast to int32
    like ``fused_sparse.py:297-298``).  Returns (B, H, T, D) in ``q.dtype``
    unless ``out_dtype`` is given.  Negative indices wrap by Tk like torch
    indexing unless ``mask_negative`` is set, in which case they are excluded
    from the softmax.  Differentiable in q, k and v when autograd records (the
    reference's gather path is too, ``fused_sparse.py:64-94``); the indices carry
    no gradient.  ``dropout_p`` > 0 drops attention probabilities like the reference's
    training path (``models/attention.py:50-54``); the mask comes from ``dropout_seed``
    (drawn from torch's generator when None) and is recomputed by the backward.
    """
    del method, config
    _check_meat_shapes(q, k, v)
    if q.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        q, k, v = q.float(), k.float(), v.float()
    if indices.dtype != torch.int32:
        indices = indices.to(torch.int32)
    if not 0.0 <= dropout_p < 1.0:
        raise ValueError(f"dropout_p must be in [0, 1), got {dropout_p}")
    seed = 0
    if dropout_p > 0.0:
        seed = int(dropout_seed) if dropout_seed is not None else int(torch.randint(0, 2 ** 62, (1,)).item())
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        if status is not None:
            raise ValueError("status is not supported on the differentiable path")
        return _SparseMeatFunction.apply(q, k, v, indices, scale, mask_negative, out_dtype, float(dropout_p), seed)
    with torch.no_grad():
        return _launch_attention(q, k, v, indices, scale, mask_negative=mask_negative, out_dtype=out_dtype,
                                 status=status, drop_rate=float(dropout_p), drop_seed=seed)


def sparse_meat_attention_reference(q, k, v, indices, scale):
    """Name kept from ``fused_sparse.py:80-94``; runs the same CUDA kernel (fp32 arithmetic)."""
    return sparse_meat_attention(q, k, v, indices, scale, method="reference")


@torch.no_grad()
def fused_sparse_attention(
    q_search: torch.Tensor,
    k_search: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    top_k: int,
    scale: float,
    *,
    retrieval_method: str = "auto",
    meat_method: str = "auto",
    meat_config: SparseMeatConfig | None = None,
    pad_mode: str = "reference",
    out_dtype: torch.dtype | None = None,
    status: torch.Tensor | None = None,
    key_mask: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Causal top-K retrieval + sparse attention: returns (out (B,H,T,D), indices (B,T,K) int32).

    Mirrors ``fused_sparse_attention`` (``routing_attention/kernels/fused_sparse.py:327-356``).
    ``pad_mode="masked"`` excludes the pad slots of rows ``i < K-1`` from the
    softmax instead of attending to them as the reference does.
    ``key_mask`` (B, T), an extension (the reference ignores padding here): padded
    keys are never retrieved and unfilled slots are masked.
    """
    del retrieval_method, meat_method, meat_config
    if q_search.shape != k_search.shape:
        raise ValueError(f"query/key shape mismatch: {q_search.shape} vs {k_search.shape}")
    if q_search.dim() != 3:
        raise ValueError(f"expected (B,T,R), got {tuple(q_search.shape)}")
    _check_meat_shapes(q, k, v)
    B, T, R = q_search.shape
    if q.shape[0] != B or q.shape[2] != T or k.shape[2] != T:
        raise ValueError(f"search vectors {tuple(q_search.shape)} do not match q/k/v {tuple(q.shape)}")
    k_eff = min(int(top_k), T)
    if k_eff <= 0:
        idx = torch.zeros(B, T, 0, dtype=torch.int32, device=q.device)
        return torch.zeros(q.shape, dtype=out_dtype or q.dtype, device=q.device), idx
    dev = _lib.require_cuda(q_search, k_search, q, k, v)
    lib = _lib.load_library()
    qa, ka, _ = promote_compute_dtype(q_search, k_search, None)
    if q.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        q, k, v = q.float(), k.float(), v.float()
    q, k, v = _attn_operand(q), _attn_operand(k), _attn_operand(v)
    H, D = q.shape[1], q.shape[3]
    idx = torch.empty(B, T, k_eff, dtype=torch.int32, device=dev)
    out = torch.empty(B, H, T, D, dtype=out_dtype or q.dtype, device=dev)
    if key_mask is not None:
        # padded keys are never retrieved; slots a row cannot fill are masked out of the softmax
        from .causal_topk import _launch_topk_key_mask

        idx = _launch_topk_key_mask(qa, ka, int(top_k), key_mask, status=status)
        out = _launch_attention(q, k, v, idx, scale, mask_negative=True, out_dtype=out_dtype, status=status)
        return out, idx
    ws = _lib.workspace(B, T, T, R, int(top_k), qa.dtype, dev)
    st = _lib.status_arg(dev, status)
    with torch.cuda.device(dev):
        rc = lib.wf_fused_sparse_attention(
            qa.data_ptr(), ka.data_ptr(), _lib.dtype_code(qa.dtype), R, _lib.strides(qa), _lib.strides(ka),
            q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q.dtype), B, H, T, T, D,
            _lib.strides(q), _lib.strides(k), _lib.strides(v), int(top_k), float(scale),
            pad_mode_code(pad_mode), 0, 1, 0, idx.data_ptr(), out.data_ptr(), _lib.dtype_code(out.dtype),
            _lib.strides(out), ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            st, _lib.stream_ptr(dev),
        )
    _lib.check(rc)
    _lib.status_after(dev, status)
    return out, idx


def fused_sparse_attention_available() -> bool:
    """True when the CUDA library is built and a GPU is visible (``fused_sparse.py:60-61``)."""
    return _lib.LIB_PATH.exists() and torch.cuda.is_available()


__all__ = [
    "SparseMeatConfig",
    "sparse_meat_attention",
    "sparse_meat_attention_reference",
    "fused_sparse_attention",
    "fused_sparse_attention_available",
    "_launch_topk",
]
