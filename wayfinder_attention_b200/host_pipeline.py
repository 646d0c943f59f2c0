"""Fused retrieval + sparse attention on host-resident tensors, with copies overlapped.

``fused_sparse_attention`` (``routing_attention/kernels/fused_sparse.py:327-356``)
takes device tensors.  A caller whose activations live in pinned host memory
would otherwise run three serial phases per call: upload q_search/k_search/q/k/v,
compute, download (out, indices).  ``HostFusedSparseAttention`` overlaps them:

  copy-in stream:   addresses | q,k,v rows of chunk 0 | chunk 1 | ... | chunk P-1
  compute stream:             top-K (all rows)  | attn 0 | attn 1 | ... | attn P-1
  copy-out stream:                     indices | out 0  | out 1  | ... | out P-1

Retrieval needs only the addresses (d_A elements per row, a few percent of the
bytes), so it runs while q/k/v are still arriving.  Attention of query rows
[a, e) reads K/V rows < e only (the indices are causal), so chunk c starts as
soon as the rows of chunks 0..c are on the device.  The device kernels and
their results are exactly those of ``fused_sparse_attention``; only the copy
schedule differs.  PCIe is full duplex, so uploads and downloads proceed
together; the call costs roughly the upload time plus one chunk of attention
and one chunk of download.  The schedule itself is native
(``wf_fused_sparse_attention_host``): one call enqueues every copy, event and
kernel, so the host adds microseconds, not a Python loop, per chunk.
"""

from __future__ import annotations

import torch

from . import _lib
from .causal_topk import pad_mode_code, promote_compute_dtype
from .fused_sparse import _check_meat_shapes


def _device_like(x: torch.Tensor, dev: torch.device) -> torch.Tensor:
    return torch.empty_strided(tuple(x.shape), tuple(x.stride()), dtype=x.dtype, device=dev)


class HostFusedSparseAttention:
    """``fused_sparse_attention`` for pinned host tensors, upload/compute/download overlapped.

    ``chunks`` is the number of query-row chunks the sequence is split into for
    the pipeline.  Device staging buffers and streams persist between calls of
    the same shapes.  With ``download_indices=False`` the retrieved indices stay on
    the device (``last_indices``) and the call returns ``(out, None)``: a third less
    to download at K=128, H*D=512.  ``__call__`` enqueues everything behind the current stream
    and makes the current stream wait for the downloads, so the host outputs are
    valid after ``torch.cuda.current_stream().synchronize()``.
    """

    def __init__(self, top_k: int, scale: float, *, chunks: int = 8, pad_mode: str = "reference",
                 device: torch.device | str | int = 0, download_indices: bool = True):
        if chunks < 1:
            raise ValueError(f"chunks must be >= 1, got {chunks}")
        self.top_k = int(top_k)
        self.scale = float(scale)
        self.chunks = int(chunks)
        self.pad_mode = pad_mode
        self.download_indices = bool(download_indices)
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self._bufs: dict[str, torch.Tensor] = {}
        self._key = None
        self._s_in = self._s_out = None
        self._ws = None
        self._ws_key = None
        self.last_indices: torch.Tensor | None = None

    def _staging(self, tensors: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        key = tuple((n, tuple(t.shape), tuple(t.stride()), t.dtype) for n, t in tensors.items())
        if key != self._key:
            self._bufs = {n: _device_like(t, self.device) for n, t in tensors.items()}
            self._key = key
        return self._bufs

    @torch.no_grad()
    def __call__(self, q_search: torch.Tensor, k_search: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                 v: torch.Tensor, out: torch.Tensor | None = None,
                 idx_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Host (B,T,R) addresses and (B,H,T,D) q/k/v in; host (out (B,H,T,D), indices (B,T,K) int32) out."""
        for name, t in (("q_search", q_search), ("k_search", k_search), ("q", q), ("k", k), ("v", v)):
            if t.is_cuda:
                raise ValueError(f"{name} must be a host tensor (use fused_sparse_attention for device tensors)")
        if q_search.shape != k_search.shape or q_search.dim() != 3:
            raise ValueError(f"expected matching (B,T,R) addresses, got {tuple(q_search.shape)}, {tuple(k_search.shape)}")
        _check_meat_shapes(q, k, v)
        B, T, R = q_search.shape
        H, D = q.shape[1], q.shape[3]
        if q.shape[0] != B or q.shape[2] != T or k.shape[2] != T:
            raise ValueError(f"search vectors {tuple(q_search.shape)} do not match q/k/v {tuple(q.shape)}")
        if q.dtype not in (torch.bfloat16, torch.float16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
            raise ValueError(f"q/k/v must share one of bf16/f16/f32, got {q.dtype}, {k.dtype}, {v.dtype}")
        k_eff = min(self.top_k, T)
        if out is None:
            out = torch.empty(B, T, H, D, dtype=q.dtype, pin_memory=True).transpose(1, 2)
        if idx_out is None and self.download_indices:
            idx_out = torch.empty(B, T, max(k_eff, 0), dtype=torch.int32, pin_memory=True)
        if tuple(out.shape) != (B, H, T, D):
            raise ValueError("out has the wrong shape")
        if idx_out is not None and (tuple(idx_out.shape) != (B, T, max(k_eff, 0)) or not idx_out.is_contiguous()
                                    or idx_out.dtype != torch.int32):
            raise ValueError(f"idx_out must be a contiguous int32 tensor of shape {(B, T, max(k_eff, 0))}")
        if k_eff <= 0 or B == 0 or H == 0:
            out.zero_()  # softmax over an empty set: the reference's sum over zero rows
            return out, idx_out
        dev = self.device
        qa_h, ka_h, _ = promote_compute_dtype(q_search, k_search, None)
        qa_h, ka_h = qa_h.contiguous(), ka_h.contiguous()
        idx_like = idx_out if idx_out is not None else torch.empty(B, T, k_eff, dtype=torch.int32)
        d = self._staging({"qa": qa_h, "ka": ka_h, "q": q, "k": k, "v": v, "out": out, "idx": idx_like})
        if self._ws is None or self._ws_key != (B, T, R, self.top_k, qa_h.dtype):
            self._ws = _lib.workspace(B, T, T, R, self.top_k, qa_h.dtype, dev)
            self._ws_key = (B, T, R, self.top_k, qa_h.dtype)
        if self._s_in is None:
            self._s_in = torch.cuda.Stream(device=dev)
            self._s_out = torch.cuda.Stream(device=dev)
        ws = self._ws
        lib = _lib.load_library()
        st = _lib.status_arg(dev, None)
        with torch.cuda.device(dev):
            rc = lib.wf_fused_sparse_attention_host(
                qa_h.data_ptr(), ka_h.data_ptr(), _lib.dtype_code(qa_h.dtype), R,
                q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q.dtype), B, H, T, D,
                _lib.strides(q), _lib.strides(k), _lib.strides(v), self.top_k, self.scale,
                pad_mode_code(self.pad_mode), min(self.chunks, T, 64),
                idx_out.data_ptr() if idx_out is not None else None, out.data_ptr(),
                _lib.dtype_code(out.dtype), _lib.strides(out),
                d["qa"].data_ptr(), d["ka"].data_ptr(), d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(),
                d["idx"].data_ptr(), d["out"].data_ptr(), ws.data_ptr() if ws is not None else None,
                ws.numel() if ws is not None else 0, st, _lib.stream_ptr(dev),
                self._s_in.cuda_stream, self._s_out.cuda_stream,
            )
        _lib.check(rc)
        _lib.status_after(dev, None)
        self.last_indices = d["idx"]
        return out, idx_out

    forward = __call__


def host_fused_sparse_attention(q_search, k_search, q, k, v, top_k: int, scale: float, *, chunks: int = 8,
                                pad_mode: str = "reference", out=None, idx_out=None):
    """One-shot form of :class:`HostFusedSparseAttention` (allocates its staging buffers per call)."""
    op = HostFusedSparseAttention(top_k, scale, chunks=chunks, pad_mode=pad_mode,
                                  device=torch.cuda.current_device())
    return op(q_search, k_search, q, k, v, out=out, idx_out=idx_out)
