"""CPU-only checks: the C-ABI library loads and exports what include/wayfinder.h declares,
argument validation fails cleanly without touching a GPU, and the host-side logic
(shape checks, sharding plans, workload arithmetic) behaves."""

import ctypes
import re

import numpy as np
import pytest
import torch

from conftest import REPO
from wayfinder_attention_b200 import _lib, causal_topk, fused_sparse_attention, sparse_meat_attention
from wayfinder_attention_b200.sharding import batch_shard, local_rows
from wayfinder_attention_b200.workloads import CONFIGS, make_inputs


def _declared_symbols():
    text = (REPO / "include" / "wayfinder.h").read_text()
    return sorted(set(re.findall(r"WF_API\s+[\w\s\*]+?\b(wf_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    declared = _declared_symbols()
    assert set(declared) >= {"wf_causal_topk", "wf_sparse_attention", "wf_fused_sparse_attention"}
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/wayfinder.h but not exported"
    assert set(_lib.EXPORTED_SYMBOLS) <= set(declared)


def test_version_and_limits():
    lib = _lib.load_library()
    assert lib.wf_version() >= 100
    assert lib.wf_max_top_k() >= 256


def _i64(*v):
    return (ctypes.c_int64 * len(v))(*v)


def test_invalid_arguments_fail_without_gpu():
    lib = _lib.load_library()
    s = _i64(1, 1, 1)
    rc = lib.wf_causal_topk(None, None, 0, 1, -5, 10, 32, s, s, 8, 0, 0, 1, 0, None, None, 0, None, None)
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT
    assert b"negative" in lib.wf_last_error()
    rc = lib.wf_causal_topk(None, None, 7, 1, 5, 10, 32, s, s, 8, 0, 0, 1, 0, None, None, 0, None, None)
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT and b"dtype" in lib.wf_last_error()
    rc = lib.wf_causal_topk(None, None, 0, 1, 5, 10, 32, s, s, 8, 9, 0, 1, 0, None, None, 0, None, None)
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT and b"pad_mode" in lib.wf_last_error()
    # empty work is a successful no-op
    rc = lib.wf_causal_topk(None, None, 0, 0, 5, 10, 32, s, s, 8, 0, 0, 1, 0, None, None, 0, None, None)
    assert rc == _lib.WF_OK
    s4 = _i64(1, 1, 1, 1)
    rc = lib.wf_sparse_attention(None, None, None, 0, None, 1, 1, 4, 4, 48, 4, s4, s4, s4, s, 1.0, 0, None, 0,
                                 s4, None, None)
    assert rc == _lib.WF_ERR_UNSUPPORTED and b"head_dim" in lib.wf_last_error()
    rc = lib.wf_sparse_attention(None, None, None, 0, None, 1, 1, 4, 4, 64, 4, s4, s4, s4, s, float("nan"), 0,
                                 None, 0, s4, None, None)
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT and b"scale" in lib.wf_last_error()
    # row map reaching beyond the keys
    rc = lib.wf_causal_topk(ctypes.c_void_p(16), ctypes.c_void_p(16), 0, 1, 128, 128, 32, s, s, 8, 0, 64, 2, 1,
                            ctypes.c_void_p(16), None, 0, None, None)
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT and b"row map" in lib.wf_last_error()
    rc = lib.wf_causal_topk(ctypes.c_void_p(16), ctypes.c_void_p(16), 0, 1, 128, 4096, 32, s, s, 300, 0, 0, 1, 0,
                            ctypes.c_void_p(16), None, 0, None, None)
    assert rc == _lib.WF_ERR_UNSUPPORTED and b"maximum" in lib.wf_last_error()


def test_host_pipeline_entry_validates_before_enqueueing():
    lib = _lib.load_library()
    p = ctypes.c_void_p(4096)
    B, H, T, D, R = 1, 2, 256, 64, 32
    rows = _i64(T * H * D, D, H * D, 1)  # (B,T,H,D)-major
    bad = _i64(T * H * D, 1, H * D, 2)   # stride(D) != 1

    def call(top_k=16, chunks=4, qs=rows):
        return lib.wf_fused_sparse_attention_host(p, p, 0, R, p, p, p, 0, B, H, T, D, qs, rows, rows, top_k, 1.0, 0,
                                                  chunks, p, p, 0, rows, p, p, p, p, p, p, p, None, 0, None, None,
                                                  None, None)

    assert call(top_k=0) == _lib.WF_ERR_INVALID_ARGUMENT and b"top_k" in lib.wf_last_error()
    assert call(chunks=0) == _lib.WF_ERR_INVALID_ARGUMENT and b"chunks" in lib.wf_last_error()
    assert call(chunks=65) == _lib.WF_ERR_INVALID_ARGUMENT
    assert call(qs=bad) == _lib.WF_ERR_UNSUPPORTED and b"stride" in lib.wf_last_error()


def test_address_projection_entry_validates_before_launch():
    lib = _lib.load_library()
    p = ctypes.c_void_p(4096)

    def call(n_out=64, group=32, d_model=256, dtype=0, xs=256):
        return lib.wf_address_projection(p, dtype, 100, d_model, xs, p, None, n_out, group, 1, p, n_out, None, None)

    assert call(group=24) == _lib.WF_ERR_INVALID_ARGUMENT and b"group" in lib.wf_last_error()
    assert call(group=64) == _lib.WF_ERR_INVALID_ARGUMENT
    assert call(n_out=48, group=16) == _lib.WF_ERR_UNSUPPORTED and b"n_out" in lib.wf_last_error()
    assert call(xs=100) == _lib.WF_ERR_INVALID_ARGUMENT and b"stride" in lib.wf_last_error()
    assert call(dtype=9) == _lib.WF_ERR_INVALID_ARGUMENT
    assert lib.wf_address_projection(None, 0, 0, 256, 256, None, None, 64, 32, 1, None, 64, None, None) == _lib.WF_OK


def test_key_mask_entry_validates_before_launch():
    lib = _lib.load_library()
    p = ctypes.c_void_p(4096)
    s = _i64(4096, 32, 1)
    ms = _i64(128, 1)
    n = lib.wf_causal_topk_key_mask_workspace_bytes(1, 128, 32, 16, 0)
    assert n > 0
    rc = lib.wf_causal_topk_key_mask(p, p, 0, 1, 128, 32, s, s, None, ms, 16, p, p, n, None, None)
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT and b"key_mask" in lib.wf_last_error()
    rc = lib.wf_causal_topk_key_mask(p, p, 0, 1, 128, 32, s, s, p, ms, 16, p, p, n - 1, None, None)
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT and b"workspace" in lib.wf_last_error()


def test_python_api_validates_like_reference():
    a = torch.zeros(1, 8, 32)
    with pytest.raises(ValueError, match="shape mismatch"):
        causal_topk(a, torch.zeros(1, 9, 32), 4)
    with pytest.raises(ValueError, match=r"expected \(B,T,R\)"):
        causal_topk(torch.zeros(8, 32), torch.zeros(8, 32), 4)
    assert causal_topk(a, a, 0).shape == (1, 8, 0)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        causal_topk(a, a, 4)
    q = torch.zeros(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        sparse_meat_attention(q, q, q, torch.zeros(1, 8, 4, dtype=torch.int32), 0.125)
    with pytest.raises(ValueError):
        sparse_meat_attention(q, q[:, :1], q, torch.zeros(1, 8, 4, dtype=torch.int32), 0.125)
    with pytest.raises(ValueError):
        fused_sparse_attention(a, a, q[:, :, :4], q, q, 4, 0.125)


def test_batch_shard_partitions():
    for B in (1, 7, 8, 64):
        for W in (1, 2, 3, 8):
            ranges = [batch_shard(B, W, r) for r in range(W)]
            assert ranges[0][0] == 0 and ranges[-1][1] == B
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(W - 1))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        batch_shard(8, 2, 2)


def test_local_rows_partition_and_balance():
    T, tile = 65536, 256
    for W in (1, 2, 4, 8):
        parts = [local_rows(T, W, r, tile) for r in range(W)]
        allrows = np.sort(np.concatenate(parts))
        assert np.array_equal(allrows, np.arange(T))
        work = [float((p + 1).sum()) for p in parts]  # causal scoring work ~ sum of positions
        assert max(work) / min(work) < 1.08  # scoring only; attention work is equal per row
    parts = [local_rows(1000, 3, r, 64) for r in range(3)]
    assert np.array_equal(np.sort(np.concatenate(parts)), np.arange(1000))
    with pytest.raises(ValueError):
        local_rows(1000, 3, 0, 100)


def test_workload_arithmetic_matches_roofline_table():
    w = CONFIGS["cfg2"]
    assert w.queries == 16384
    assert abs(w.score_flops() - 8.59e9) / 8.59e9 < 0.01
    assert abs(w.gathered_bytes() - 4.29e9) / 4.29e9 < 0.01
    w4 = CONFIGS["cfg4"]
    assert abs(w4.gathered_bytes() - 1.37e11) / 1.37e11 < 0.01


def test_synthetic_inputs_are_seeded_and_laid_out_like_the_module():
    w = CONFIGS["cfg1"]
    a = make_inputs(w)
    b = make_inputs(w)
    for k in a:
        assert torch.equal(a[k], b[k])
    assert a["q"].shape == (1, 4, 2048, 64) and a["q"].transpose(1, 2).is_contiguous()
    assert abs(a["q_addr"].float().std().item() - 32 ** -0.5) < 0.01


def test_workspace_query():
    lib = _lib.load_library()
    assert lib.wf_causal_topk_workspace_bytes(1, 16384, 16384, 32, 128, _lib.WF_DTYPE_BF16) == 16384 * (4 * 256 * 8 + 16)
    assert lib.wf_causal_topk_workspace_bytes(2, 100, 100, 32, 64, _lib.WF_DTYPE_F16) == 200 * (4 * 256 * 8 + 16)
    # fp32 addresses: the lists plus bf16 copies of the query and key addresses
    assert lib.wf_causal_topk_workspace_bytes(1, 2048, 2048, 32, 128, _lib.WF_DTYPE_F32) == (
        2048 * (4 * 256 * 8 + 16) + (2048 + 2048) * 32 * 2 + 256)
    # K <= 256 on tensor cores: lists of 384 slots above K = 128
    assert lib.wf_causal_topk_workspace_bytes(1, 2048, 2048, 32, 256, _lib.WF_DTYPE_BF16) == 2048 * (4 * 384 * 8 + 16)
    # large batches run in slices of 65536 // T batch elements that reuse one workspace
    assert lib.wf_causal_topk_workspace_bytes(64, 8192, 8192, 32, 128, _lib.WF_DTYPE_BF16) == 8 * 8192 * (4 * 256 * 8 + 16)
    assert lib.wf_causal_topk_workspace_bytes(1, 65536, 65536, 32, 128, _lib.WF_DTYPE_BF16) == 65536 * (4 * 256 * 8 + 16)
    assert lib.wf_causal_topk_workspace_bytes(1, 2048, 2048, 32, 300, _lib.WF_DTYPE_BF16) == 0  # CUDA-core path
