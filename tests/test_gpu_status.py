"""Kernel faults that do not stop a kernel reach the caller as exceptions.

A bounded wait of the tensor-core retrieval is made to run out without any GPU
fault: the library's test hook has one CTA of each pair withhold its arrive on the
peer's barrier of one bisection exchange, and bounds that wait at 2 ms.  The
waiting CTA must give up, drain what it issued, free its tensor memory and return
with the status word set; the context stays usable and the next call is exact.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

WAIT_NS = 2_000_000


def _addresses(T, R, seed):
    g = torch.Generator().manual_seed(seed)
    qa = (torch.randn(1, T, R, generator=g) / R ** 0.5).to(torch.bfloat16)
    ka = (torch.randn(1, T, R, generator=g) / R ** 0.5).to(torch.bfloat16)
    return qa.cuda(), ka.cuda()


def test_timeout_sets_the_callers_status_word(cuda_device):
    from wayfinder_attention_b200 import _lib, causal_topk

    qa, ka = _addresses(256, 32, 5)
    good = causal_topk(qa, ka, 16)
    lib = _lib.load_library()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    assert lib.wf_testing_withhold_pair_arrive(0, WAIT_NS) == 0
    causal_topk(qa, ka, 16, status=status)
    torch.cuda.synchronize()
    bits = int(status.item())
    assert bits & _lib.STATUS_WAIT_TIMEOUT, hex(bits)
    assert bits & 256, hex(bits)  # the wait site: a bisection exchange with the peer CTA
    again = causal_topk(qa, ka, 16)  # the hook is one-shot and the context is intact
    _lib.check_status()
    assert torch.equal(again, good)


def test_timeout_raises_without_a_status_word(cuda_device):
    from wayfinder_attention_b200 import _lib, causal_topk, check_status, fused_sparse_attention

    qa, ka = _addresses(384, 32, 6)
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 2, 384, 64, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    ref_out, ref_idx = fused_sparse_attention(qa, ka, q, k, v, 32, 0.125)
    check_status()
    lib = _lib.load_library()
    assert lib.wf_testing_withhold_pair_arrive(3, WAIT_NS) == 0
    causal_topk(qa, ka, 32)
    with pytest.raises(RuntimeError, match="timed out"):
        check_status()
    check_status()  # the word was cleared when it was reported
    out, idx = fused_sparse_attention(qa, ka, q, k, v, 32, 0.125)
    check_status()
    assert torch.equal(idx, ref_idx) and torch.equal(out, ref_out)


def test_out_of_range_index_raises_at_check(cuda_device):
    from wayfinder_attention_b200 import check_status, sparse_meat_attention

    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(1, 2, 64, 32, generator=g).cuda() for _ in range(3))
    idx = torch.zeros(1, 64, 4, dtype=torch.int32)
    idx[0, 5, 1] = 64  # one past the last key
    check_status()
    out = sparse_meat_attention(q, k, v, idx.cuda(), 0.2)
    with pytest.raises(RuntimeError, match="out of range"):
        check_status()
    assert torch.isnan(out[0, :, 5]).all() and not torch.isnan(out[0, :, 4]).any()
    check_status()


def test_fault_surfaces_at_a_later_call_without_check(cuda_device):
    """Without check_status the fault still reaches the caller: the first launch after
    a read-back interval queues the status copy, and the call after it raises."""
    from wayfinder_attention_b200 import _lib, check_status, sparse_meat_attention

    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 64, 32, generator=g).cuda() for _ in range(3))
    good = torch.zeros(1, 64, 4, dtype=torch.int32, device="cuda")
    bad = good.clone()
    bad[0, 7, 0] = -1000  # below -Tk: out of range
    check_status()
    sparse_meat_attention(q, k, v, bad, 0.2)
    with pytest.raises(RuntimeError, match="out of range"):
        for _ in range(2 * _lib.READBACK_CALLS + 2):
            sparse_meat_attention(q, k, v, good, 0.2)
            torch.cuda.synchronize()
    check_status()
