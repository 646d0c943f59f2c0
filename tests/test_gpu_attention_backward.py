"""Backward of the sparse attention (wf_sparse_attention_backward) against autograd.

The reference for every case is PyTorch autograd through the gather formulation of
the reference's sparse attention (routing_attention/kernels/fused_sparse.py:64-94,
the path its non-fused training uses, models/attention.py:35-56) evaluated in fp64
on the same (dtype-rounded) inputs.  Tolerances: fp32 gradients within 1e-5 of the
gradient's scale; 16-bit gradients (accumulated in fp32, rounded once) within one
ulp of that type plus 1e-5 of the scale.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(q, k, v, idx, scale, mask_negative, dout):
    q, k, v = (x.double().detach().requires_grad_(True) for x in (q, k, v))
    Tk = k.shape[2]
    il = idx.long()
    valid = il >= 0 if mask_negative else torch.ones_like(il, dtype=torch.bool)
    ic = torch.where(valid, il % Tk, torch.zeros_like(il))
    B, H, T, D = q.shape
    bidx = torch.arange(B, device=q.device)[:, None, None]
    ksel = k.permute(0, 2, 1, 3)[bidx, ic]  # (B, T, K, H, D)
    vsel = v.permute(0, 2, 1, 3)[bidx, ic]
    s = torch.einsum("bhtd,btkhd->bhtk", q, ksel) * scale
    s = s.masked_fill(~valid[:, None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    out = torch.einsum("bhtk,btkhd->bhtd", p, vsel)
    out.backward(dout.double())
    return out.detach(), q.grad, k.grad, v.grad


def _close(got, want, dtype):
    got, want = got.double(), want.double()
    scale = want.abs().max().item() + 1e-30
    if dtype == torch.float32:
        return (got - want).abs().max().item() <= 1e-5 * scale
    mant = {torch.bfloat16: 7, torch.float16: 10}[dtype]
    ulp = torch.exp2(torch.floor(torch.log2(want.abs().clamp_min(1e-30))) - mant)
    return bool(((got - want).abs() <= ulp + 1e-5 * scale).all())


def _case(B, H, Tq, Tk, D, K, dtype, layout, mask_negative, duplicates, seed, dev):
    g = torch.Generator().manual_seed(seed)
    shape_q, shape_kv = (B, Tq, H, D), (B, Tk, H, D)
    q = torch.randn(shape_q, generator=g).to(dtype)
    k = torch.randn(shape_kv, generator=g).to(dtype)
    v = torch.randn(shape_kv, generator=g).to(dtype)
    if layout == "bthd":  # the module's views: (B, H, T, D) over (B, T, H, D) memory
        q, k, v = (x.transpose(1, 2) for x in (q, k, v))
    else:
        q, k, v = (x.transpose(1, 2).contiguous() for x in (q, k, v))
    if duplicates:
        idx = torch.randint(0, Tk, (B, Tq, K), generator=g, dtype=torch.int32)
    else:
        idx = torch.stack([torch.stack([torch.randperm(Tk, generator=g)[:K] for _ in range(Tq)]) for _ in range(B)])
        idx = idx.to(torch.int32)
    if mask_negative:
        drop = torch.rand(B, Tq, K, generator=g) < 0.2
        drop[..., 0] = False  # every row keeps at least one key
        idx = torch.where(drop, torch.full_like(idx, -1), idx)
    dout = torch.randn(B, H, Tq, D, generator=g).to(dtype)
    return q.to(dev), k.to(dev), v.to(dev), idx.to(dev), dout.to(dev)


@pytest.mark.parametrize("B,H,Tq,Tk,D,K,dtype,layout,mask_negative,duplicates", [
    (2, 4, 300, 300, 64, 32, torch.float32, "bthd", False, False),
    (1, 8, 257, 700, 64, 48, torch.float32, "bhtd", True, False),   # Tq != Tk, masked slots
    (2, 2, 200, 200, 32, 16, torch.float32, "bthd", False, True),   # duplicate indices add up
    (1, 8, 512, 512, 64, 128, torch.bfloat16, "bthd", False, False),  # cfg2-like head layout
    (1, 4, 300, 300, 128, 64, torch.float16, "bthd", True, True),
    (3, 1, 100, 100, 32, 8, torch.bfloat16, "bhtd", False, True),
])
def test_backward_matches_autograd(B, H, Tq, Tk, D, K, dtype, layout, mask_negative, duplicates, cuda_device):
    from wayfinder_attention_b200 import sparse_meat_attention

    q, k, v, idx, dout = _case(B, H, Tq, Tk, D, K, dtype, layout, mask_negative, duplicates, Tq + K, cuda_device)
    scale = D ** -0.5
    qg, kg, vg = (x.detach().clone().requires_grad_(True) for x in (q, k, v))
    out = sparse_meat_attention(qg, kg, vg, idx, scale, mask_negative=mask_negative)
    out.backward(dout)
    want_out, dq, dk, dv = _reference(q, k, v, idx, scale, mask_negative, dout)
    assert qg.grad.dtype == dtype and qg.grad.shape == q.shape
    assert _close(qg.grad, dq, dtype), "dq"
    assert _close(kg.grad, dk, dtype), "dk"
    assert _close(vg.grad, dv, dtype), "dv"


def test_backward_keys_nobody_retrieved_get_zero(cuda_device):
    from wayfinder_attention_b200 import sparse_meat_attention

    q, k, v, idx, dout = _case(1, 2, 64, 256, 64, 8, torch.float32, "bthd", False, False, 3, cuda_device)
    idx = idx % 100  # keys 100..255 are never retrieved
    kg, vg = k.detach().clone().requires_grad_(True), v.detach().clone().requires_grad_(True)
    sparse_meat_attention(q, kg, vg, idx, 0.125).backward(dout)
    assert torch.count_nonzero(kg.grad[:, :, 100:]) == 0 and torch.count_nonzero(vg.grad[:, :, 100:]) == 0
    assert torch.count_nonzero(kg.grad[:, :, :100]) > 0


def test_module_trains_through_the_sparse_path(cuda_device):
    """LearnedAddressSparseAttention (non-fused path, no probability dropout): one optimizer step
    with gradients for the q/k/v/out projections from the CUDA backward."""
    from wayfinder_attention_b200 import LearnedAddressSparseAttention

    torch.manual_seed(11)
    m = LearnedAddressSparseAttention(128, 2, top_k=16, dropout=0.0,
                                      retrieval_config={"use_fused_sparse": False}).to(cuda_device).train()
    x = torch.randn(2, 128, 128, device=cuda_device)
    target = torch.randn(2, 128, 128, device=cuda_device)
    opt = torch.optim.SGD(m.parameters(), lr=0.1)
    losses = []
    for _ in range(3):
        opt.zero_grad()
        loss = ((m(x) - target) ** 2).mean()
        loss.backward()
        losses.append(loss.item())
        for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
            gw = getattr(m, name).weight.grad
            assert gw is not None and torch.isfinite(gw).all() and gw.abs().sum() > 0, name
        opt.step()
    assert losses[-1] < losses[0]


def _keep_mask(seed, B, H, T, K, rate):
    """The kernels' keep decisions, recomputed in numpy (SplitMix64 output function of
    seed + (idx + 1) * 0x9E3779B97F4A7C15, 24 high bits, keep when u >= rate)."""
    import numpy as np

    idx = np.arange(B * H * T * K, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (idx + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    u = (z >> np.uint64(40)).astype(np.float64) / 16777216.0
    return torch.from_numpy((u >= float(np.float32(rate))).reshape(B, H, T, K))


def _reference_dropout(q, k, v, idx, scale, dout, keep, rate):
    q, k, v = (x.double().detach().requires_grad_(True) for x in (q, k, v))
    Tk = k.shape[2]
    ic = idx.long() % Tk
    B = q.shape[0]
    bidx = torch.arange(B, device=q.device)[:, None, None]
    ksel = k.permute(0, 2, 1, 3)[bidx, ic]
    vsel = v.permute(0, 2, 1, 3)[bidx, ic]
    p = torch.softmax(torch.einsum("bhtd,btkhd->bhtk", q, ksel) * scale, dim=-1)
    p = p * keep.to(p.device, p.dtype) / (1.0 - rate)
    out = torch.einsum("bhtk,btkhd->bhtd", p, vsel)
    out.backward(dout.double())
    return out.detach(), q.grad, k.grad, v.grad


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_dropout_forward_and_backward_match_autograd(dtype, cuda_device):
    from wayfinder_attention_b200 import sparse_meat_attention

    B, H, T, D, K, rate, seed = 2, 4, 300, 64, 32, 0.25, 123456789
    q, k, v, idx, dout = _case(B, H, T, T, D, K, dtype, "bthd", False, False, 77, cuda_device)
    keep = _keep_mask(seed, B, H, T, K, rate)
    assert abs(1.0 - keep.float().mean().item() - rate) < 0.01
    qg, kg, vg = (x.detach().clone().requires_grad_(True) for x in (q, k, v))
    out = sparse_meat_attention(qg, kg, vg, idx, D ** -0.5, dropout_p=rate, dropout_seed=seed)
    out.backward(dout)
    want_out, dq, dk, dv = _reference_dropout(q, k, v, idx, D ** -0.5, dout, keep, rate)
    assert _close(out.detach(), want_out, dtype), "out"
    assert _close(qg.grad, dq, dtype), "dq"
    assert _close(kg.grad, dk, dtype), "dk"
    assert _close(vg.grad, dv, dtype), "dv"
    # the no-grad forward draws the same mask from the same seed
    with torch.no_grad():
        again = sparse_meat_attention(q, k, v, idx, D ** -0.5, dropout_p=rate, dropout_seed=seed)
    assert torch.equal(again, out.detach())


def test_module_trains_with_attention_dropout(cuda_device):
    from wayfinder_attention_b200 import LearnedAddressSparseAttention

    torch.manual_seed(12)
    m = LearnedAddressSparseAttention(128, 2, top_k=16, dropout=0.1,
                                      retrieval_config={"use_fused_sparse": False}).to(cuda_device).train()
    x = torch.randn(2, 128, 128, device=cuda_device)
    # a target the layer can move toward quickly (its output norm), so the trend is
    # far larger than the step-to-step noise of the dropout masks
    target = torch.zeros(2, 128, 128, device=cuda_device)
    opt = torch.optim.SGD(m.parameters(), lr=0.5)
    losses = []
    for _ in range(6):
        opt.zero_grad()
        loss = ((m(x) - target) ** 2).mean()
        loss.backward()
        losses.append(loss.item())
        opt.step()
    assert losses[-1] < losses[0]
    m.eval()
    with torch.no_grad():
        assert torch.equal(m(x), m(x))  # no dropout in eval mode
