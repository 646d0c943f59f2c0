"""HostFusedSparseAttention: host tensors in and out, copies overlapped with the kernels.

The device kernels are the ones ``fused_sparse_attention`` runs, so the host
pipeline must reproduce its outputs bit for bit, for any chunking and for both
host memory layouts of q/k/v/out; the oracle pins the small case.
"""

import numpy as np
import pytest
import torch

from parity_utils import compare_indices, oracle

pytestmark = pytest.mark.gpu


def _inputs(B, H, T, D, R, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    qa = (torch.randn(B, T, R, generator=g) / R ** 0.5).to(dtype)
    ka = (torch.randn(B, T, R, generator=g) / R ** 0.5).to(dtype)
    qkv = [torch.randn(B, T, H, D, generator=g).to(dtype) for _ in range(3)]
    return qa, ka, qkv


@pytest.mark.parametrize("chunks", [1, 3, 8])
@pytest.mark.parametrize("layout", ["bthd", "bhtd"])
def test_host_pipeline_matches_device_call(chunks, layout):
    from wayfinder_attention_b200 import HostFusedSparseAttention, fused_sparse_attention

    B, H, T, D, R, K = 2, 4, 1000, 64, 32, 64
    qa, ka, qkv = _inputs(B, H, T, D, R, torch.bfloat16, 7 + chunks)
    if layout == "bthd":
        q, k, v = (x.pin_memory().transpose(1, 2) for x in qkv)
    else:
        q, k, v = (x.transpose(1, 2).contiguous().pin_memory() for x in qkv)
    qa_p, ka_p = qa.pin_memory(), ka.pin_memory()
    scale = D ** -0.5
    op = HostFusedSparseAttention(K, scale, chunks=chunks, device=0)
    for _ in range(2):  # second call reuses the staging buffers
        out_h, idx_h = op(qa_p, ka_p, q, k, v)
        torch.cuda.current_stream().synchronize()
    ref_out, ref_idx = fused_sparse_attention(qa.cuda(), ka.cuda(), q.cuda(), k.cuda(), v.cuda(), K, scale)
    assert not out_h.is_cuda and not idx_h.is_cuda
    assert torch.equal(idx_h, ref_idx.cpu())
    assert torch.equal(out_h, ref_out.cpu())


@pytest.mark.parametrize("shape", [(2, 4, 1000, 64, 64, 8), (1, 4, 2048, 64, 128, 8), (1, 2, 200, 32, 128, 4),
                                   (1, 2, 512, 32, 16, 64)])
def test_host_pipeline_first_call_on_poisoned_staging(shape, monkeypatch):
    """The first call must not read staging rows before their upload lands.

    Rows i < K-1 attend their pad rows (i + K + s + 1) % T, up to row 3K-2 and
    wrapping when 3K-2 >= T, so they need later chunks than their own.  The device
    staging buffers start as NaN (indices as garbage): any K/V row read before its
    copy landed shows up as a NaN or a mismatch on the very first call.
    """
    from wayfinder_attention_b200 import HostFusedSparseAttention, fused_sparse_attention
    from wayfinder_attention_b200 import host_pipeline

    def poisoned(x, dev):
        t = torch.empty_strided(tuple(x.shape), tuple(x.stride()), dtype=x.dtype, device=dev)
        if t.dtype.is_floating_point:
            t.fill_(float("nan"))
        else:
            t.fill_(-12345)
        return t

    monkeypatch.setattr(host_pipeline, "_device_like", poisoned)
    B, H, T, D, K, chunks = shape
    qa, ka, qkv = _inputs(B, H, T, D, 32, torch.bfloat16, 11)
    q, k, v = (x.pin_memory().transpose(1, 2) for x in qkv)
    scale = D ** -0.5
    op = HostFusedSparseAttention(K, scale, chunks=chunks, device=0)
    torch.cuda.synchronize()
    out_h, idx_h = op(qa.pin_memory(), ka.pin_memory(), q, k, v)
    torch.cuda.current_stream().synchronize()
    ref_out, ref_idx = fused_sparse_attention(qa.cuda(), ka.cuda(), q.cuda(), k.cuda(), v.cuda(), K, scale)
    assert torch.equal(idx_h, ref_idx.cpu())
    assert not torch.isnan(out_h).any()
    assert torch.equal(out_h, ref_out.cpu())


def test_host_pipeline_against_oracle_and_outputs_given():
    from wayfinder_attention_b200 import host_fused_sparse_attention

    B, H, T, D, R, K = 1, 2, 300, 32, 32, 16
    qa, ka, qkv = _inputs(B, H, T, D, R, torch.float32, 3)
    q, k, v = (x.pin_memory().transpose(1, 2) for x in qkv)
    out_h = torch.full((B, H, T, D), float("nan")).pin_memory()
    idx_h = torch.full((B, T, K), -7, dtype=torch.int32).pin_memory()
    scale = 0.3
    out, idx = host_fused_sparse_attention(qa.pin_memory(), ka.pin_memory(), q, k, v, K, scale, chunks=4,
                                           out=out_h, idx_out=idx_h)
    torch.cuda.synchronize()
    assert out is out_h and idx is idx_h
    o_ref, i_ref = oracle.fused_sparse_attention(qa.numpy(), ka.numpy(), q.numpy(), k.numpy(), v.numpy(), K, scale)
    assert not compare_indices(idx.numpy(), i_ref, qa.numpy(), ka.numpy())["bad"]
    np.testing.assert_allclose(out.numpy(), o_ref, rtol=1e-5, atol=1e-5)


def test_host_pipeline_without_index_download():
    from wayfinder_attention_b200 import HostFusedSparseAttention, fused_sparse_attention

    B, H, T, D, R, K = 1, 4, 1500, 64, 32, 64
    qa, ka, qkv = _inputs(B, H, T, D, R, torch.bfloat16, 21)
    q, k, v = (x.pin_memory().transpose(1, 2) for x in qkv)
    op = HostFusedSparseAttention(K, D ** -0.5, chunks=4, device=0, download_indices=False)
    out_h, idx_h = op(qa.pin_memory(), ka.pin_memory(), q, k, v)
    torch.cuda.current_stream().synchronize()
    assert idx_h is None and op.last_indices.is_cuda
    ref_out, ref_idx = fused_sparse_attention(qa.cuda(), ka.cuda(), q.cuda(), k.cuda(), v.cuda(), K, D ** -0.5)
    assert torch.equal(op.last_indices, ref_idx)
    assert torch.equal(out_h, ref_out.cpu())


def test_host_pipeline_rejects_device_inputs():
    from wayfinder_attention_b200 import HostFusedSparseAttention

    qa, ka, qkv = _inputs(1, 2, 64, 32, 32, torch.float32, 1)
    op = HostFusedSparseAttention(8, 1.0)
    with pytest.raises(ValueError):
        op(qa.cuda(), ka, *(x.transpose(1, 2) for x in qkv))
