"""The sequence-sharded attention kernels on one GPU, with the ranks emulated.

Each emulated rank's K/V buffers are built locally exactly as the all-gathers of
``SequenceShardedAttention`` lay them out (rank-major, or chunk-major for the
chunked form), so the key-position -> (chunk, rank, row) arithmetic of
``wf_sparse_attention_cyclic_kv[_chunked]`` is checked bit for bit against the
single-GPU fused call without a second GPU or any collective.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(B, T, H, D, R, seed):
    g = torch.Generator().manual_seed(seed)
    qa = (torch.randn(B, T, R, generator=g) / R ** 0.5).bfloat16().cuda()
    ka = (torch.randn(B, T, R, generator=g) / R ** 0.5).bfloat16().cuda()
    qkv = [torch.randn(B, T, H, D, generator=g).bfloat16().cuda() for _ in range(3)]  # (B, T, H, D) memory
    return qa, ka, qkv


@pytest.mark.parametrize("B,T,H,D,K,world,tile,chunks,pad_mode", [
    (2, 4096, 4, 64, 128, 4, 256, 2, "reference"),
    (1, 4096, 8, 64, 128, 2, 256, 8, "reference"),
    (2, 2048, 2, 128, 64, 8, 128, 2, "masked"),
    (1, 8192, 4, 64, 128, 8, 256, 4, "reference"),
])
def test_chunked_cyclic_kv_matches_single_gpu(B, T, H, D, K, world, tile, chunks, pad_mode):
    from wayfinder_attention_b200 import fused_sparse_attention
    from wayfinder_attention_b200.sharding import chunked_kv_attention, local_rows, sharded_causal_topk

    qa, ka, (q, k, v) = _case(B, T, H, D, 32, 40 + world)
    full_out, full_idx = fused_sparse_attention(qa, ka, q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                K, D ** -0.5, pad_mode=pad_mode)
    Tl = T // world
    Tc = Tl // chunks
    rows = [torch.from_numpy(local_rows(T, world, r, tile)).cuda() for r in range(world)]
    # what the chunked all-gathers leave on every rank: block (c, w) = rank w's local rows of chunk c
    k_g = torch.stack([torch.stack([k[:, rows[w][c * Tc:(c + 1) * Tc]] for w in range(world)]) for c in range(chunks)])
    v_g = torch.stack([torch.stack([v[:, rows[w][c * Tc:(c + 1) * Tc]] for w in range(world)]) for c in range(chunks)])
    for r in range(world):
        idx = sharded_causal_topk(qa[:, rows[r]].contiguous(), ka, K, world, r, tile, pad_mode)
        assert torch.equal(idx, full_idx[:, rows[r]])
        q_l = q[:, rows[r]].contiguous().transpose(1, 2)
        out = chunked_kv_attention(q_l, idx, k_g, v_g, D ** -0.5, tile, pad_mode)
        assert torch.equal(out, full_out[:, :, rows[r]]), f"rank {r}"


@pytest.mark.parametrize("world", [2, 4])
def test_rank_major_cyclic_kv_matches_single_gpu(world):
    from wayfinder_attention_b200 import _lib, fused_sparse_attention
    from wayfinder_attention_b200.sharding import local_rows

    B, T, H, D, K, tile = 2, 2048, 4, 64, 64, 128
    qa, ka, (q, k, v) = _case(B, T, H, D, 32, 7)
    full_out, full_idx = fused_sparse_attention(qa, ka, q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                K, D ** -0.5)
    rows = [torch.from_numpy(local_rows(T, world, r, tile)).cuda() for r in range(world)]
    k_g = torch.stack([k[:, rows[w]] for w in range(world)])  # (W, B, Tl, H, D): one all-gather
    v_g = torch.stack([v[:, rows[w]] for w in range(world)])
    kb, vb = k_g[0].permute(0, 2, 1, 3), v_g[0].permute(0, 2, 1, 3)
    lib = _lib.load_library()
    for r in range(world):
        qc = q[:, rows[r]].contiguous().transpose(1, 2)
        ic = full_idx[:, rows[r]].contiguous()
        out = torch.empty_like(qc)
        rc = lib.wf_sparse_attention_cyclic_kv(
            qc.data_ptr(), kb.data_ptr(), vb.data_ptr(), _lib.WF_DTYPE_BF16, ic.data_ptr(), B, H, qc.shape[2], T, D,
            K, _lib.strides(qc), _lib.strides(kb), _lib.strides(vb), _lib.strides(ic), D ** -0.5, 0, out.data_ptr(),
            _lib.WF_DTYPE_BF16, _lib.strides(out), tile, world, k_g.stride(0), v_g.stride(0), None,
            _lib.stream_ptr(qc.device))
        _lib.check(rc)
        assert torch.equal(out, full_out[:, :, rows[r]]), f"rank {r}"
