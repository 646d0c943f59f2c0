"""The operators replay from a CUDA graph: a captured decoder prefill and a captured
fused op equal their eager calls bit for bit, on new inputs after capture."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_captured_decoder_prefill_equals_eager(cuda_device):
    from wayfinder_attention_b200 import CapturedForward, TransformerLM, check_status

    torch.manual_seed(0)
    lm = TransformerLM(128, d_model=128, n_layers=2, n_heads=2, d_ff=256, max_seq_len=1024, dropout=0.0,
                       attention_type="learned_address", routing_top_k=64,
                       retrieval_config={"use_fused_sparse": True, "method": "fused_causal"})
    lm = lm.to(cuda_device, torch.bfloat16).eval()
    g = torch.Generator(device=cuda_device).manual_seed(1)
    ids0 = torch.randint(0, 128, (2, 1024), device=cuda_device, generator=g)
    cap = CapturedForward(lambda ids: lm(ids)["logits"], ids0)
    for _ in range(2):
        ids = torch.randint(0, 128, (2, 1024), device=cuda_device, generator=g)
        got = cap(ids).clone()
        with torch.no_grad():
            want = lm(ids)["logits"]
        assert torch.equal(got, want)
    check_status()


def test_captured_fused_op_equals_eager(cuda_device):
    from wayfinder_attention_b200 import CapturedForward, fused_sparse_attention

    g = torch.Generator(device=cuda_device).manual_seed(2)

    def inputs():
        qa = (torch.randn(1, 2048, 32, device=cuda_device, generator=g) / 32 ** 0.5).bfloat16()
        ka = (torch.randn(1, 2048, 32, device=cuda_device, generator=g) / 32 ** 0.5).bfloat16()
        q, k, v = (torch.randn(1, 4, 2048, 64, device=cuda_device, generator=g).bfloat16() for _ in range(3))
        return qa, ka, q, k, v

    cap = CapturedForward(lambda *x: fused_sparse_attention(*x, 128, 0.125), *inputs())
    x = inputs()
    out, idx = cap(*x)
    want_out, want_idx = fused_sparse_attention(*x, 128, 0.125)
    assert torch.equal(idx, want_idx) and torch.equal(out, want_out)
