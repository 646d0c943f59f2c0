"""Retrieval that skips padded keys (wf_causal_topk_key_mask) and its fused / module use.

The oracle (``oracle.causal_topk_key_mask``) ranks, for query t, the keys j <= t that
the (B, T) padding mask keeps, by fp32 score with ties to the lower index; unfilled
slots are -1.  Index rows must match it exactly except where the K-th and (K+1)-th
candidates' fp64 scores differ by less than 1e-6 relative (the repository's
near-tie rule).
"""

import numpy as np
import pytest
import torch

from parity_utils import oracle

pytestmark = pytest.mark.gpu


def _masks(B, T, g):
    random = (torch.rand(B, T, generator=g) < 0.7)
    left = torch.ones(B, T, dtype=torch.bool)
    left[:, : T // 3] = False  # left padding: early rows see no key at all
    right = torch.ones(B, T, dtype=torch.bool)
    right[:, T - T // 4:] = False
    return {"random": random, "left": left, "right": right}


def _check(got, want, q, k, mask):
    got, want = got.cpu().numpy(), np.asarray(want)
    bad = []
    # slot order within a row is unspecified: compare the rows as sets (-1 tails included)
    for b, t in zip(*np.nonzero((np.sort(got, axis=-1) != np.sort(want, axis=-1)).any(-1))):
        valid = np.nonzero(mask[b].numpy())[0]
        cand = valid[valid <= t]
        s = k[b, cand].double().numpy() @ q[b, t].double().numpy()
        srt = np.sort(s)[::-1]
        K = got.shape[-1]
        if cand.size <= K or abs(srt[K - 1] - srt[K]) >= 1e-6 * abs(srt[K - 1]):
            bad.append((int(b), int(t)))
    assert not bad, f"{len(bad)} rows differ, first {bad[:5]}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("kind", ["random", "left", "right"])
def test_key_mask_matches_oracle(dtype, kind, cuda_device):
    from wayfinder_attention_b200 import causal_topk

    B, T, R, K = 2, 700, 32, 64
    g = torch.Generator().manual_seed(T + K)
    q = (torch.randn(B, T, R, generator=g) / R ** 0.5).to(dtype)
    k = (torch.randn(B, T, R, generator=g) / R ** 0.5).to(dtype)
    mask = _masks(B, T, g)[kind]
    got = causal_topk(q.to(cuda_device), k.to(cuda_device), K, key_mask=mask.to(cuda_device))
    want = oracle.causal_topk_key_mask(q.float().numpy(), k.float().numpy(), K, mask.numpy())
    _check(got, want, q.float(), k.float(), mask)
    gi = got.cpu()
    # properties on every row: padded keys never retrieved, causal, -1 only as a tail
    valid_idx = gi >= 0
    assert bool((gi[valid_idx] < T).all())
    b_ix = torch.arange(B)[:, None, None].expand_as(gi)
    assert bool(mask[b_ix[valid_idx], gi[valid_idx].long()].all())
    assert bool((gi <= torch.arange(T)[None, :, None]).all())
    assert bool((valid_idx[..., 1:] <= valid_idx[..., :-1]).all())


def test_all_ones_mask_equals_plain_retrieval_with_masked_pads(cuda_device):
    from wayfinder_attention_b200 import causal_topk

    B, T, R, K = 2, 1500, 32, 128
    g = torch.Generator().manual_seed(9)
    q = (torch.randn(B, T, R, generator=g) / R ** 0.5).to(torch.bfloat16).to(cuda_device)
    k = (torch.randn(B, T, R, generator=g) / R ** 0.5).to(torch.bfloat16).to(cuda_device)
    ones = torch.ones(B, T, dtype=torch.bool, device=cuda_device)
    assert torch.equal(causal_topk(q, k, K, key_mask=ones), causal_topk(q, k, K, pad_mode="masked"))


def test_fused_with_key_mask_against_oracle(cuda_device):
    from wayfinder_attention_b200 import fused_sparse_attention

    B, H, T, D, R, K = 1, 4, 400, 64, 32, 32
    g = torch.Generator().manual_seed(21)
    qa = torch.randn(B, T, R, generator=g) / R ** 0.5
    ka = torch.randn(B, T, R, generator=g) / R ** 0.5
    q, k, v = (torch.randn(B, H, T, D, generator=g) for _ in range(3))
    mask = _masks(B, T, g)["random"]
    out, idx = fused_sparse_attention(qa.to(cuda_device), ka.to(cuda_device), q.to(cuda_device), k.to(cuda_device),
                                      v.to(cuda_device), K, D ** -0.5, key_mask=mask.to(cuda_device))
    want_idx = oracle.causal_topk_key_mask(qa.numpy(), ka.numpy(), K, mask.numpy())
    _check(idx, want_idx, qa, ka, mask)
    rows = np.nonzero(mask[0].numpy().cumsum() > 0)[0]  # rows that see at least one key
    want = oracle.sparse_meat_attention(q.numpy(), k.numpy(), v.numpy(), idx.cpu().numpy(), D ** -0.5,
                                        mask_negative=True)
    np.testing.assert_allclose(out.cpu().numpy()[:, :, rows], want[:, :, rows], rtol=1e-5, atol=1e-5)


def test_module_honours_attn_mask_when_asked(cuda_device):
    from wayfinder_attention_b200 import LearnedAddressSparseAttention

    torch.manual_seed(4)
    m = LearnedAddressSparseAttention(128, 2, top_k=16, mask_padded_keys=True,
                                      retrieval_config={"use_fused_sparse": True}).to(cuda_device).eval()
    x = torch.randn(2, 200, 128, device=cuda_device)
    pad = torch.ones(2, 200, dtype=torch.bool, device=cuda_device)
    pad[1, :50] = False  # left padding of the second sequence
    with torch.no_grad():
        y_masked = m(x, attn_mask=pad)
        # changing padded positions must not change the outputs of the real tokens
        x2 = x.clone()
        x2[1, :50] = torch.randn_like(x2[1, :50])
        y2 = m(x2, attn_mask=pad)
        m.mask_padded_keys = False
        y_plain = m(x, attn_mask=pad)
        y_plain2 = m(x2, attn_mask=pad)
    assert torch.allclose(y_masked[1, 50:], y2[1, 50:], atol=1e-6)
    assert not torch.allclose(y_plain[1, 50:], y_plain2[1, 50:], atol=1e-6)  # the reference behaviour leaks
    # the unpadded sequence: same as without the mask on rows with a full candidate set
    assert torch.allclose(y_masked[0, 15:], y_plain[0, 15:], atol=1e-6)
