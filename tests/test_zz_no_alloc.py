"""The allocation-free retrieval entry point, called through the C ABI.

Some callers cannot allocate device memory (no allocator of their own, or a
context where cudaMalloc is off limits), so wf_causal_topk_noalloc draws its
scratch from a fixed array inside the library.  Two calls in a row, on different
inputs, must both return exactly what wf_causal_topk returns with a workspace; a
request larger than the built-in array must be refused cleanly.  This file is
collected last so that a failure here never hides the other tests.
"""

import ctypes

import pytest
import torch

from wayfinder_attention_b200 import _lib, causal_topk
from wayfinder_attention_b200.workloads import Workload, make_inputs, to_device

pytestmark = pytest.mark.gpu


def _noalloc(lib):
    f = lib.wf_causal_topk_noalloc
    f.restype = ctypes.c_int
    vp, i32, i64, i64p = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)
    f.argtypes = [vp, vp, i32, i64, i64, i64, i32, i64p, i64p, i32, i32, i32, i32, i32, vp, vp, vp]
    return f


def _call(f, qa, ka, K, out, status, dev):
    B, T, R = qa.shape
    return f(qa.data_ptr(), ka.data_ptr(), _lib.dtype_code(qa.dtype), B, T, T, R, _lib.strides(qa),
             _lib.strides(ka), K, _lib.WF_PAD_REFERENCE, 0, 1, 0, out.data_ptr(), status.data_ptr(),
             _lib.stream_ptr(dev))


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    lib = _lib.load_library()
    f = _noalloc(lib)
    K = 128
    # the second call reuses the array left by the first; fp32 addresses also keep
    # bf16 copies of the address rows in the array, so fewer rows fit (2012 at R=32)
    for seed, T, dt in ((45, 2000, torch.bfloat16), (46, 1200, torch.bfloat16), (47, 2012, torch.float32)):
        w = Workload("t", 1, 1, T, 16, 32, K, dt)
        x = to_device(make_inputs(w, seed=seed), cuda_device)
        got = torch.full((1, T, K), -7, dtype=torch.int32, device=cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        rc = _call(f, x["q_addr"], x["k_addr"], K, got, status, cuda_device)
        assert rc == _lib.WF_OK, lib.wf_last_error()
        want = causal_topk(x["q_addr"], x["k_addr"], K)  # the workspace entry point
        torch.cuda.synchronize()
        assert status.item() == 0
        assert torch.equal(got, want)


def test_noalloc_rejects_requests_beyond_its_array(cuda_device):
    lib = _lib.load_library()
    f = _noalloc(lib)
    T, K = 16384, 128
    w = Workload("t", 1, 1, T, 16, 32, K, torch.bfloat16)
    x = to_device(make_inputs(w), cuda_device)
    out = torch.empty(1, T, K, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rc = _call(f, x["q_addr"], x["k_addr"], K, out, status, cuda_device)
    assert rc == _lib.WF_ERR_UNSUPPORTED
    assert b"built-in" in lib.wf_last_error()
    # fp32 addresses: 2013 rows no longer fit beside their bf16 copies
    w = Workload("t", 1, 1, 2013, 16, 32, K, torch.float32)
    x = to_device(make_inputs(w), cuda_device)
    out = torch.empty(1, 2013, K, dtype=torch.int32, device=cuda_device)
    assert _call(f, x["q_addr"], x["k_addr"], K, out, status, cuda_device) == _lib.WF_ERR_UNSUPPORTED
