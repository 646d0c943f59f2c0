"""ctypes binding of libwayfinder_sm100.so (the C ABI in include/wayfinder.h).

Only plain pointers, sizes and strides cross this boundary.  The library must
exist next to this file (built by ``wayfinder_attention_b200.build``); there
is no fallback implementation, so a missing library raises immediately.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

import os

# WF_LIB_PATH points at an alternative build of the same library (e.g. an instrumented one).
LIB_PATH = Path(os.environ.get("WF_LIB_PATH") or Path(__file__).resolve().parent / "libwayfinder_sm100.so")

WF_DTYPE_BF16 = 0
WF_DTYPE_F16 = 1
WF_DTYPE_F32 = 2

WF_OK = 0
WF_ERR_INVALID_ARGUMENT = 1
WF_ERR_UNSUPPORTED = 2
WF_ERR_CUDA = 3

WF_PAD_REFERENCE = 0
WF_PAD_MASKED = 1
WF_ATTN_MASK_NEGATIVE = 1

EXPORTED_SYMBOLS = (
    "wf_version",
    "wf_last_error",
    "wf_max_top_k",
    "wf_causal_topk_workspace_bytes",
    "wf_causal_topk",
    "wf_sparse_attention",
    "wf_sparse_attention_cyclic_kv",
    "wf_fused_sparse_attention",
    "wf_fused_sparse_attention_host",
    "wf_address_projection",
    "wf_sparse_attention_backward",
    "wf_sparse_attention_backward_workspace_bytes",
    "wf_causal_topk_key_mask",
    "wf_causal_topk_key_mask_workspace_bytes",
    "wf_sparse_attention_dropout",
    "wf_sparse_attention_cyclic_kv_chunked",
)

_DTYPE_CODES = {
    torch.bfloat16: WF_DTYPE_BF16,
    torch.float16: WF_DTYPE_F16,
    torch.float32: WF_DTYPE_F32,
}

_lib = None
_lock = threading.Lock()

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_i64p = ctypes.POINTER(ctypes.c_int64)


def _declare(lib: ctypes.CDLL) -> None:
    lib.wf_version.restype = ctypes.c_int
    lib.wf_version.argtypes = []
    lib.wf_last_error.restype = ctypes.c_char_p
    lib.wf_last_error.argtypes = []
    lib.wf_max_top_k.restype = ctypes.c_int
    lib.wf_max_top_k.argtypes = []
    lib.wf_causal_topk.restype = ctypes.c_int
    lib.wf_causal_topk.argtypes = [
        _vp, _vp, _i32, _i64, _i64, _i64, _i32, _i64p, _i64p, _i32, _i32, _i32, _i32, _i32, _vp,
        _vp, ctypes.c_size_t, _vp, _vp,
    ]
    lib.wf_causal_topk_workspace_bytes.restype = ctypes.c_size_t
    lib.wf_causal_topk_workspace_bytes.argtypes = [_i64, _i64, _i64, _i32, _i32, _i32]
    lib.wf_sparse_attention.restype = ctypes.c_int
    lib.wf_sparse_attention.argtypes = [
        _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i32, _i32,
        _i64p, _i64p, _i64p, _i64p, _f32, _i32, _vp, _i32, _i64p, _vp, _vp,
    ]
    lib.wf_sparse_attention_cyclic_kv.restype = ctypes.c_int
    lib.wf_sparse_attention_cyclic_kv.argtypes = [
        _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i32, _i32,
        _i64p, _i64p, _i64p, _i64p, _f32, _i32, _vp, _i32, _i64p, _i32, _i32, _i64, _i64, _vp, _vp,
    ]
    lib.wf_sparse_attention_cyclic_kv_chunked.restype = ctypes.c_int
    lib.wf_sparse_attention_cyclic_kv_chunked.argtypes = [
        _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i32, _i32,
        _i64p, _i64p, _i64p, _i64p, _f32, _i32, _vp, _i32, _i64p, _i32, _i32, _i32, _i64, _i64, _vp, _vp,
    ]
    lib.wf_fused_sparse_attention.restype = ctypes.c_int
    lib.wf_fused_sparse_attention.argtypes = [
        _vp, _vp, _i32, _i32, _i64p, _i64p,
        _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32,
        _i64p, _i64p, _i64p, _i32, _f32, _i32, _i32, _i32, _i32,
        _vp, _vp, _i32, _i64p, _vp, ctypes.c_size_t, _vp, _vp,
    ]
    lib.wf_fused_sparse_attention_host.restype = ctypes.c_int
    lib.wf_fused_sparse_attention_host.argtypes = [
        _vp, _vp, _i32, _i32, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i32, _i64p, _i64p, _i64p,
        _i32, _f32, _i32, _i32, _vp, _vp, _i32, _i64p,
        _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp, _vp, _vp, _vp,
    ]
    lib.wf_address_projection.restype = ctypes.c_int
    lib.wf_address_projection.argtypes = [
        _vp, _i32, _i64, _i32, _i64, _vp, _vp, _i32, _i32, _i32, _vp, _i64, _vp, _vp,
    ]
    lib.wf_sparse_attention_backward_workspace_bytes.restype = ctypes.c_size_t
    lib.wf_sparse_attention_backward_workspace_bytes.argtypes = [_i64, _i64, _i64, _i64, _i32]
    lib.wf_sparse_attention_backward.restype = ctypes.c_int
    lib.wf_sparse_attention_backward.argtypes = [
        _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _i64p, _i64p, _i64p, _i64p,
        _vp, _i64p, _f32, _i32, _f32, ctypes.c_uint64, _vp, _vp, _vp, _i32, _i64p, _i64p, _i64p, _vp,
        ctypes.c_size_t, _vp, _vp,
    ]
    lib.wf_sparse_attention_dropout.restype = ctypes.c_int
    lib.wf_sparse_attention_dropout.argtypes = [
        _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _i64p, _i64p, _i64p, _i64p, _f32, _i32,
        _f32, ctypes.c_uint64, _vp, _i32, _i64p, _vp, _vp,
    ]
    lib.wf_causal_topk_key_mask_workspace_bytes.restype = ctypes.c_size_t
    lib.wf_causal_topk_key_mask_workspace_bytes.argtypes = [_i64, _i64, _i32, _i32, _i32]
    lib.wf_causal_topk_key_mask.restype = ctypes.c_int
    lib.wf_causal_topk_key_mask.argtypes = [
        _vp, _vp, _i32, _i64, _i64, _i32, _i64p, _i64p, _vp, _i64p, _i32, _vp, _vp, ctypes.c_size_t, _vp, _vp,
    ]


def load_library() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"wayfinder CUDA library not found at {LIB_PATH}; build it with "
                    "`python -m wayfinder_attention_b200.build` (there is no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            _declare(lib)
            _lib = lib
    return _lib


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; expected bfloat16, float16 or float32") from None


def strides(t: torch.Tensor):
    arr = (ctypes.c_int64 * t.dim())(*t.stride())
    return arr


def check(rc: int) -> None:
    """Map a C-ABI return code to the reference's exception types."""
    if rc == WF_OK:
        return
    msg = load_library().wf_last_error().decode("utf-8", "replace")
    if rc in (WF_ERR_INVALID_ARGUMENT, WF_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def workspace(B: int, Tq: int, Tk: int, R: int, top_k: int, dtype: torch.dtype, device) -> torch.Tensor | None:
    """Scratch the retrieval kernel needs (None if none), from torch's caching allocator."""
    n = load_library().wf_causal_topk_workspace_bytes(B, Tq, Tk, R, top_k, dtype_code(dtype))
    if n == 0:
        return None
    return torch.empty(n, dtype=torch.uint8, device=device)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                "wayfinder_attention_b200 runs on CUDA tensors only (no CPU fallback); "
                f"got a tensor on {t.device}"
            )
        if t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev
