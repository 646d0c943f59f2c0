"""ctypes binding of libwayfinder_sm100.so (the C ABI in include/wayfinder.h).

Only plain pointers, sizes and strides cross this boundary.  The library must
exist next to this file (built by ``wayfinder_attention_b200.build``); there
is no fallback implementation, so a missing library raises immediately.
"""

from __future__ import annotations

import ctypes
import os
import threading
import time
from pathlib import Path

import torch

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
    "wf_causal_topk_noalloc",
    "wf_testing_withhold_pair_arrive",
    "wf_gather_rows_bench",
    "wf_gather_rows_bulk_bench",
    "wf_peer_buffer_alloc",
    "wf_peer_buffer_free",
    "wf_peer_buffer_open",
    "wf_peer_buffer_close",
    "wf_pack_row_blocks",
    "wf_peer_pull_blocks",
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
    lib.wf_peer_buffer_alloc.restype = ctypes.c_int
    lib.wf_peer_buffer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]
    lib.wf_peer_buffer_free.restype = ctypes.c_int
    lib.wf_peer_buffer_free.argtypes = [_vp]
    lib.wf_peer_buffer_open.restype = ctypes.c_int
    lib.wf_peer_buffer_open.argtypes = [_vp, ctypes.POINTER(_vp)]
    lib.wf_peer_buffer_close.restype = ctypes.c_int
    lib.wf_peer_buffer_close.argtypes = [_vp]
    lib.wf_pack_row_blocks.restype = ctypes.c_int
    lib.wf_pack_row_blocks.argtypes = [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _i64, _i64, _i32, _vp]
    lib.wf_peer_pull_blocks.restype = ctypes.c_int
    lib.wf_peer_pull_blocks.argtypes = [ctypes.POINTER(_vp), _i32, _i32, _i32, _i32, _i64, _i64, _i64, _i64, _vp,
                                        ctypes.POINTER(_vp), _i32, ctypes.POINTER(_vp)]
    lib.wf_gather_rows_bulk_bench.restype = ctypes.c_int
    lib.wf_gather_rows_bulk_bench.argtypes = [_vp, _vp, _i64, _vp, _i64, _i32, _i64, _i32, _vp, _vp]
    lib.wf_gather_rows_bench.restype = ctypes.c_int
    lib.wf_gather_rows_bench.argtypes = [_vp, _vp, _i64, _i64, _vp, _i64, _i32, _i64, _vp, _vp]
    lib.wf_testing_withhold_pair_arrive.restype = ctypes.c_int
    lib.wf_testing_withhold_pair_arrive.argtypes = [_i32, ctypes.c_uint64]
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


# ---------------------------------------------------------------- status word
# Every kernel reports faults it can detect without stopping (an out-of-range
# attention index: bit 0; a bounded wait that gave up: bit 1, plus a bit naming the
# wait site from bit 4 up) by OR-ing bits into a caller-provided int32 status word.
# A caller that passes none gets this per-device word.  Its value is copied
# asynchronously into pinned host memory after a launch — after the first launch,
# then at most every READBACK_CALLS launches or READBACK_SECONDS, so the copy costs
# nothing measurable — and a later call on the device raises ``RuntimeError`` once
# that copy has landed.  ``check_status`` copies, waits and raises at once.  No
# call synchronises the host except ``check_status``.  Launches captured into a CUDA
# graph write the same word when the graph replays; it is read back by the next
# eager call or by ``check_status``.

STATUS_INDEX_OUT_OF_RANGE = 1
STATUS_WAIT_TIMEOUT = 2
READBACK_CALLS = 64
READBACK_SECONDS = 0.05


class _DeviceStatus:
    def __init__(self, dev: torch.device):
        self.dev = dev
        self.word = torch.zeros(1, dtype=torch.int32, device=dev)
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = torch.cuda.Event()
        self.pending = False
        self.calls = 0
        self.last = float("-inf")

    def poll(self, wait: bool = False) -> None:
        if wait:
            self.readback()
        if not self.pending:
            return
        if wait:
            self.event.synchronize()
        elif not self.event.query():
            return
        self.pending = False
        bits = int(self.host[0])
        if bits:
            with torch.cuda.device(self.dev):
                self.word.zero_()
            raise RuntimeError(describe_status(bits))

    def readback(self) -> None:
        with torch.cuda.device(self.dev):
            self.host.copy_(self.word, non_blocking=True)
            self.event.record()
        self.pending = True
        self.calls = 0
        self.last = time.monotonic()

    def after_launch(self) -> None:
        self.calls += 1
        if self.pending:
            return  # the last read-back has not been looked at yet
        if self.calls >= READBACK_CALLS or time.monotonic() - self.last >= READBACK_SECONDS:
            self.readback()


_status: dict[int, _DeviceStatus] = {}


def describe_status(bits: int) -> str:
    parts = []
    if bits & STATUS_INDEX_OUT_OF_RANGE:
        parts.append("an attention index was out of range (its output row is NaN)")
    if bits & STATUS_WAIT_TIMEOUT:
        parts.append(f"a kernel's bounded wait timed out (wait-site bits 0x{bits >> 4:x}); its results are invalid")
    if not parts:
        parts.append("unknown fault")
    return f"wayfinder kernel status 0x{bits:x}: " + "; ".join(parts)


def _device_status(dev: torch.device) -> _DeviceStatus:
    i = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _status.get(i)
    if st is None:
        st = _status[i] = _DeviceStatus(torch.device("cuda", i))
    return st


def status_arg(dev: torch.device, user: torch.Tensor | None):
    """Status pointer for a launch: the caller's word, else this device's internal one.

    Raises the fault a previous call on ``dev`` left in the internal word, if its
    read-back has landed.
    """
    if user is not None:
        if user.dtype != torch.int32 or not user.is_cuda:
            raise ValueError("status must be an int32 CUDA tensor")
        return user.data_ptr()
    st = _device_status(dev)
    if not torch.cuda.is_current_stream_capturing():  # no event queries inside a graph capture
        st.poll()
    return st.word.data_ptr()


def status_after(dev: torch.device, user: torch.Tensor | None) -> None:
    """Queue the read-back of the internal status word after a launch that used it."""
    if user is None and not torch.cuda.is_current_stream_capturing():
        _device_status(dev).after_launch()


def check_status(device=None) -> None:
    """Wait for the last calls on ``device`` (default: all used devices) and raise on any fault.

    ``RuntimeError`` names the fault; the word is cleared, so later calls run normally.
    """
    if device is None:
        targets = list(_status.values())
    else:
        d = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        targets = [_device_status(d)]
    for st in targets:
        st.poll(wait=True)
