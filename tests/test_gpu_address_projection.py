"""wf_address_projection: the fused query/key address projection + L2 normalisation.

Compared with the reference arithmetic of ``LearnedAddressModule.forward_query_key``
(``learned_address.py:39-46``: nn.Linear then F.normalize) evaluated in fp32 on the
same (dtype-rounded) inputs: within one ulp of the output type (none for fp32) plus
2^-20 of sum_d |x_d w_d| (the fp32 accumulation error; the kernel accumulates and
normalises in fp32 and rounds once).
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _within(got, want, scale, dtype):
    """|err| <= one ulp of want in the output type (none for fp32) + 2^-20 * scale.

    ``scale`` is sum_d |x_d w_d| + |b| (divided by the address norm when normalised):
    the fp32 accumulation error grows with it, not with the (possibly cancelling) result.
    """
    got, want = got.double(), want.double()
    if dtype == torch.float32:
        ulp = torch.zeros_like(want)
    else:
        mant = {torch.bfloat16: 7, torch.float16: 10}[dtype]
        ulp = torch.exp2(torch.floor(torch.log2(want.abs().clamp_min(torch.finfo(dtype).tiny))) - mant)
    return bool(((got - want).abs() <= ulp + 2.0 ** -20 * scale).all())


def _scale(x, w, b, group, normalize):
    s = F.linear(x.double().abs(), w.double().abs(), None if b is None else b.double().abs())
    if normalize:
        y = F.linear(x.double(), w.double(), None if b is None else b.double())
        norms = torch.cat([c.norm(dim=-1, keepdim=True).expand_as(c) for c in y.split(group, dim=-1)], dim=-1)
        s = s / norms.clamp_min(1e-12)
    return s


def _ref(x, w, b, group, normalize):
    y = F.linear(x.double(), w.double(), None if b is None else b.double())
    if normalize:
        y = torch.cat([F.normalize(c, dim=-1) for c in y.split(group, dim=-1)], dim=-1)
    return y


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("M,d_model,n_out,group", [
    (1000, 256, 64, 32),    # asymmetric d_A = 32: both addresses at once (tcgen05 for 16-bit inputs)
    (4096, 128, 32, 32),    # symmetric
    (300, 512, 128, 64 // 2),  # four 32-wide addresses
    (257, 100, 64, 32),     # d_model not a multiple of 8: CUDA-core form
    (64, 64, 16, 16),       # narrow addresses: CUDA-core form
])
@pytest.mark.parametrize("with_bias", [True, False])
def test_projection_matches_fp32_reference(dtype, M, d_model, n_out, group, with_bias, cuda_device):
    from wayfinder_attention_b200.address_projection import address_projection

    g = torch.Generator().manual_seed(M + d_model)
    x = torch.randn(M, d_model, generator=g).to(dtype)
    w = (torch.randn(n_out, d_model, generator=g) / d_model ** 0.5).to(dtype)
    b = (torch.randn(n_out, generator=g) * 0.1).to(dtype) if with_bias else None
    got = address_projection(x.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device),
                             group).cpu()
    want = _ref(x, w, b, group, True)
    assert _within(got, want, _scale(x, w, b, group, True), dtype)


def test_projection_without_normalisation_and_strided_rows(cuda_device):
    from wayfinder_attention_b200.address_projection import address_projection

    g = torch.Generator().manual_seed(5)
    wide = torch.randn(2, 333, 384, generator=g).to(torch.bfloat16)
    x = wide[..., :256]  # rows of 384 elements, 256 used
    w = (torch.randn(64, 256, generator=g) / 16).to(torch.bfloat16)
    b = torch.randn(64, generator=g).to(torch.bfloat16)
    got = address_projection(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), 32, normalize=False).cpu()
    want = _ref(x, w, b, 32, False)
    assert got.shape == (2, 333, 64)
    assert _within(got, want, _scale(x, w, b, 32, False), torch.bfloat16)


@pytest.mark.parametrize("similarity", ["asymmetric", "symmetric"])
def test_module_fused_projection_equals_pytorch_layers(similarity, cuda_device):
    from wayfinder_attention_b200 import LearnedAddressModule

    torch.manual_seed(7)
    m = LearnedAddressModule(256, 32, similarity=similarity).to(cuda_device).to(torch.bfloat16)
    x = torch.randn(2, 500, 256, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad():
        q, k = m.forward_query_key(x)  # fused kernel
        m.fused_projection = False
        q_ref, k_ref = m.forward_query_key(x.float().to(torch.bfloat16))
        m.fused_projection = True
        wq, bq = m.q_addr_proj.weight, m.q_addr_proj.bias
        qf = _ref(x, wq, bq, 32, True)
        qs = _scale(x, wq, bq, 32, True)
    assert q.shape == (2, 500, 32) and k.shape == (2, 500, 32)
    if similarity == "symmetric":
        assert k.data_ptr() == q.data_ptr()
    # within one bf16 ulp of the fp32 result (the PyTorch bf16 layers round twice)
    assert _within(q.float(), qf, qs, torch.bfloat16)
    assert (q.float() - q_ref.float()).abs().max().item() <= 2 ** -6
    # with gradients enabled the module keeps the PyTorch layers (autograd)
    x.requires_grad_(True)
    q2, _ = m.forward_query_key(x)
    assert q2.requires_grad
