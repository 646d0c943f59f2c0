"""Exact causal top-K retrieval over address vectors, on the sm_100a kernel.

Drop-in for ``routing_attention.kernels.causal_topk`` of the reference
(``routing_attention/kernels/causal_topk.py:470-521``).  Every ``method`` the
reference accepts computes the same exact causal top-K, so ``method`` and
``prefer_triton`` are accepted and ignored: there is one backend, the CUDA
library, and no fallback.

Output contract (identical to the reference's ``fused_causal`` path up to the
order of slots inside a row):
  * ``(B, T, K_eff)`` int32 with ``K_eff = min(top_k, T)``;
  * row ``i`` holds the ``K_eff`` keys ``j <= i`` with the largest fp32 score
    ``<q_i, k_j>`` (equal scores break to the lower key index); the order of
    those keys within the row is unspecified, as the reference's
    ``torch.topk(sorted=False)`` leaves it, but deterministic;
  * rows ``i < K_eff - 1`` have only ``i + 1`` causal keys; their remaining
    slots ``s`` hold the pad index ``(i + K_eff + s + 1) % T`` of
    ``_finalize_causal_topk`` (``causal_topk.py:37-57``), or ``-1`` with
    ``pad_mode="masked"``.
"""

from __future__ import annotations

import torch

from . import _lib

_PAD_MODES = {"reference": _lib.WF_PAD_REFERENCE, "masked": _lib.WF_PAD_MASKED}


def promote_compute_dtype(
    q: torch.Tensor, k: torch.Tensor, dtype: str | None = None
) -> tuple[torch.Tensor, torch.Tensor, torch.dtype]:
    """Dtype policy of ``routing_attention/kernels/_common.py:14-31``.

    An explicit ``dtype`` string rounds the addresses to that type first (the
    kernel then scores the rounded values exactly in fp32, as the reference's
    row-blocked path upcasts at ``causal_topk.py:150-151``); otherwise
    bf16/fp16 stay and everything else becomes fp32.
    """
    if dtype == "float16":
        target = torch.float16
    elif dtype == "bfloat16":
        target = torch.bfloat16
    elif dtype == "float32":
        target = torch.float32
    elif q.dtype in (torch.float16, torch.bfloat16):
        target = q.dtype
    else:
        target = torch.float32
    return q.to(target), k.to(target), target


def pad_mode_code(pad_mode: str) -> int:
    try:
        return _PAD_MODES[pad_mode]
    except KeyError:
        raise ValueError(f"unknown pad_mode {pad_mode!r}; expected 'reference' or 'masked'") from None


def _launch_topk(
    q: torch.Tensor,
    k: torch.Tensor,
    top_k: int,
    pad_mode: str,
    row_tile: int = 0,
    row_stride: int = 1,
    row_start: int = 0,
    out: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Run ``wf_causal_topk`` on (B, Tq, R) queries against (B, Tk, R) keys."""
    dev = _lib.require_cuda(q, k)
    lib = _lib.load_library()
    B, Tq, R = q.shape
    Tk = k.shape[1]
    k_eff = min(int(top_k), Tk)
    if out is None:
        out = torch.empty(B, Tq, max(k_eff, 0), dtype=torch.int32, device=dev)
    elif out.dtype != torch.int32 or not out.is_contiguous() or tuple(out.shape) != (B, Tq, k_eff):
        raise ValueError(f"out must be a contiguous int32 tensor of shape {(B, Tq, k_eff)}")
    ws = _lib.workspace(B, Tq, Tk, R, int(top_k), q.dtype, dev)
    st = _lib.status_arg(dev, status)
    with torch.cuda.device(dev):
        rc = lib.wf_causal_topk(
            q.data_ptr(), k.data_ptr(), _lib.dtype_code(q.dtype), B, Tq, Tk, R,
            _lib.strides(q), _lib.strides(k), int(top_k), pad_mode_code(pad_mode),
            int(row_tile), int(row_stride), int(row_start), out.data_ptr(),
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            st, _lib.stream_ptr(dev),
        )
    _lib.check(rc)
    _lib.status_after(dev, status)
    return out


@torch.no_grad()
def causal_topk(
    query: torch.Tensor,
    key: torch.Tensor,
    top_k: int,
    *,
    method: str = "auto",
    dtype: str | None = None,
    prefer_triton: bool = False,
    pad_mode: str = "reference",
    status: torch.Tensor | None = None,
    key_mask: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal top-K retrieval: (B, T, R) x (B, T, R) -> (B, T, min(top_k, T)) int32.

    Mirrors ``causal_topk`` (``routing_attention/kernels/causal_topk.py:470-521``),
    including its ``ValueError`` messages for mismatched or non-3-D inputs.
    ``key_mask`` (B, T), an extension: only keys with a nonzero mask are retrieved,
    and slots a row cannot fill are -1 (masked pads) whatever ``pad_mode`` says.
    """
    del method, prefer_triton  # one exact backend
    if query.shape != key.shape:
        raise ValueError(f"query/key shape mismatch: {query.shape} vs {key.shape}")
    if query.dim() != 3:
        raise ValueError(f"expected (B,T,R), got {tuple(query.shape)}")
    B, T, _ = query.shape
    k_eff = min(int(top_k), T)
    if k_eff == 0:
        return torch.zeros(B, T, 0, dtype=torch.int32, device=query.device)
    _lib.require_cuda(query, key)
    q, k, _ = promote_compute_dtype(query, key, dtype)
    if key_mask is not None:
        return _launch_topk_key_mask(q, k, top_k, key_mask, status=status)
    return _launch_topk(q, k, top_k, pad_mode, status=status)


def _launch_topk_key_mask(q: torch.Tensor, k: torch.Tensor, top_k: int, key_mask: torch.Tensor,
                          status: torch.Tensor | None = None) -> torch.Tensor:
    """``wf_causal_topk_key_mask``: top-K over the keys ``key_mask`` (B, T) keeps."""
    dev = _lib.require_cuda(q, k, key_mask)
    lib = _lib.load_library()
    B, T, R = q.shape
    if tuple(key_mask.shape) != (B, T):
        raise ValueError(f"key_mask must have shape {(B, T)}, got {tuple(key_mask.shape)}")
    m = key_mask.to(torch.uint8)
    k_eff = min(int(top_k), T)
    out = torch.empty(B, T, k_eff, dtype=torch.int32, device=dev)
    n = lib.wf_causal_topk_key_mask_workspace_bytes(B, T, R, int(top_k), _lib.dtype_code(q.dtype))
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=dev)
    st = _lib.status_arg(dev, status)
    with torch.cuda.device(dev):
        rc = lib.wf_causal_topk_key_mask(
            q.data_ptr(), k.data_ptr(), _lib.dtype_code(q.dtype), B, T, R, _lib.strides(q), _lib.strides(k),
            m.data_ptr(), _lib.strides(m), int(top_k), out.data_ptr(), ws.data_ptr(), ws.numel(),
            st, _lib.stream_ptr(dev),
        )
    _lib.check(rc)
    _lib.status_after(dev, status)
    return out


def causal_topk_reference(query: torch.Tensor, key: torch.Tensor, top_k: int) -> torch.Tensor:
    """Name kept from ``causal_topk.py:60-72`` (the brute-force method); same exact result here."""
    return causal_topk(query, key, top_k, method="brute_force")


def causal_topk_available() -> bool:
    """True when the CUDA library is built and a GPU is visible (``causal_topk.py:33-34``)."""
    return _lib.LIB_PATH.exists() and torch.cuda.is_available()
