"""The torch restatement of the reference's CPU execution (the timed CPU baseline)
agrees with the numpy oracle and with the reference's own golden outputs."""

import numpy as np
import torch

from parity_utils import compare_indices, load_golden, oracle

from oracle import reference_torch


def test_matches_numpy_oracle_on_sampled_rows():
    g = torch.Generator().manual_seed(9)
    B, H, T, D, R, K = 1, 2, 700, 32, 32, 48
    qa = torch.randn(B, T, R, generator=g) / R ** 0.5
    ka = torch.randn(B, T, R, generator=g) / R ** 0.5
    q, k, v = (torch.randn(B, H, T, D, generator=g) for _ in range(3))
    rows = torch.tensor([0, 5, 46, 47, 100, 333, 699])
    out, idx = reference_torch.fused_sparse_attention(qa, ka, q, k, v, K, 0.2, rows)
    want = oracle.causal_topk(qa.numpy(), ka.numpy(), K, rows=rows.numpy())
    res = compare_indices(idx.numpy(), want, qa.numpy(), ka.numpy(), rows=rows.numpy())
    assert not res["bad"]
    # attention on the restatement's own indices, against the oracle's arithmetic
    o2 = oracle.sparse_meat_attention(q.numpy(), k.numpy(), v.numpy(), idx.numpy(), 0.2, rows=rows.numpy())
    np.testing.assert_allclose(out.numpy(), o2, rtol=1e-5, atol=1e-5)


def test_matches_reference_golden():
    g = load_golden("small_f32")
    qa, ka = torch.from_numpy(g["q_addr"]), torch.from_numpy(g["k_addr"])
    K = int(g["K"])
    idx = reference_torch.causal_topk(qa, ka, K)
    res = compare_indices(idx.numpy(), g["idx"], g["q_addr"], g["k_addr"])
    assert not res["bad"]
