"""GPU parity: the sm_100a kernels (through the C ABI) against the oracle and the reference's golden outputs.

Tolerances: indices bit-exact as sets (near-tie exemption |s - s_K| <= 1e-6 |s_K|,
counted); attention output 1e-5 max-abs for fp32 arithmetic on fp32 outputs,
2e-3 max-abs for bf16 configs measured on an fp32 output buffer, and at most
one bf16 ulp for the bf16 output itself.
"""

import math

import numpy as np
import pytest
import torch

from parity_utils import compare_indices, load_golden, oracle, reference_pads, same_selection
from wayfinder_attention_b200 import causal_topk, fused_sparse_attention, sparse_meat_attention
from wayfinder_attention_b200.workloads import CONFIGS, Workload, make_inputs, scaled, to_device

pytestmark = pytest.mark.gpu

GOLDEN = ["small_f32", "short_seq", "clustered_ties", "bf16_t1024", "cfg1"]


def _golden_inputs(g, dev):
    if "q_addr" in g:
        t = {k: torch.from_numpy(g[k]) for k in ("q_addr", "k_addr", "q", "k", "v")}
    else:
        dt = getattr(torch, str(g["dtype"]))
        w = Workload("g", int(g["B"]), int(g["H"]), int(g["T"]), int(g["D"]), int(g["R"]), int(g["K"]), dt,
                     clustered=bool(g["clustered"]))
        t = make_inputs(w, seed=int(g["seed"]))
    return to_device(t, dev), {k: v.float().contiguous().numpy() for k, v in t.items()}


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("name", GOLDEN)
def test_topk_matches_reference_golden(name, cuda_device):
    g = load_golden(name)
    x, xn = _golden_inputs(g, cuda_device)
    K = int(g["K"])
    idx = causal_topk(x["q_addr"], x["k_addr"], K)
    torch.cuda.synchronize()
    got = idx.cpu().numpy()
    assert got.shape == g["idx"].shape
    res = compare_indices(got, g["idx"], xn["q_addr"], xn["k_addr"])
    assert not res["bad"], f"{len(res['bad'])} rows differ, first {res['bad'][:5]}"
    # against the oracle too (same pad convention, so pad slots must match exactly)
    want = oracle.causal_topk(xn["q_addr"], xn["k_addr"], K)
    res2 = compare_indices(got, want, xn["q_addr"], xn["k_addr"])
    assert not res2["bad"]
    T, Ke = int(g["T"]), min(K, int(g["T"]))
    for i in range(min(Ke - 1, T)):
        assert got[0, i, i + 1:].tolist() == reference_pads(i, Ke, T)


@pytest.mark.parametrize("name", GOLDEN)
def test_attention_matches_reference_golden(name, cuda_device):
    """Fed the reference's own indices, the kernel reproduces the reference output."""
    g = load_golden(name)
    x, _ = _golden_inputs(g, cuda_device)
    idx = torch.from_numpy(g["idx"]).to(cuda_device)
    out = sparse_meat_attention(x["q"], x["k"], x["v"], idx, float(g["scale"]), out_dtype=torch.float32)
    rows = torch.from_numpy(g["out_rows"]).to(cuda_device)
    got = _np(out[:, :, rows])
    err = np.abs(got - g["out"]).max()
    assert err <= 1e-5, err
    if x["q"].dtype == torch.bfloat16:
        ob = sparse_meat_attention(x["q"], x["k"], x["v"], idx, float(g["scale"]))
        assert ob.dtype == torch.bfloat16
        ref = torch.from_numpy(g["out"]).to(cuda_device)
        ulp = torch.finfo(torch.bfloat16).eps * ref.abs().clamp_min(2.0 ** -126)
        assert ((ob[:, :, rows].float() - ref).abs() <= ulp * 1.0 + 1e-6).all()


@pytest.mark.parametrize("name", ["small_f32", "cfg1", "bf16_t1024"])
def test_fused_matches_reference_golden(name, cuda_device):
    g = load_golden(name)
    x, xn = _golden_inputs(g, cuda_device)
    K = int(g["K"])
    out, idx = fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], K, float(g["scale"]),
                                      out_dtype=torch.float32)
    rows = g["out_rows"]
    got = _np(out)[:, :, rows]
    keep = rows >= K - 1
    tol = 1e-5 if x["q"].dtype == torch.float32 else 2e-3
    assert np.abs(got[:, :, keep] - g["out"][:, :, keep]).max() <= tol
    # pad rows: the oracle fed the kernel's own indices (pins numerics independently of pad slots)
    pad_rows = rows[~keep]
    if pad_rows.size:
        want = oracle.sparse_meat_attention(xn["q"], xn["k"], xn["v"], idx.cpu().numpy()[:, pad_rows],
                                            float(g["scale"]), rows=pad_rows)
        assert np.abs(got[:, :, ~keep] - want).max() <= 1e-5


def _full_scale_rows(T, K, n=384):
    rng = np.random.default_rng(7)
    return np.unique(np.concatenate([np.arange(K + 2), rng.choice(T, n, replace=False), np.arange(T - 64, T)]))


@pytest.mark.parametrize("cfg", ["cfg2"])
def test_cfg2_full_size_sampled_rows(cfg, cuda_device):
    """Headline config at full size: sampled rows against the oracle, all rows through properties."""
    w = CONFIGS[cfg]
    inp = make_inputs(w)
    x = to_device(inp, cuda_device)
    xn = {k: v.float().contiguous().numpy() for k, v in inp.items()}
    out, idx = fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], w.K, w.D ** -0.5,
                                      out_dtype=torch.float32)
    torch.cuda.synchronize()
    rows = _full_scale_rows(w.T, w.K)
    got_idx = idx.cpu().numpy()
    want_idx = oracle.causal_topk(xn["q_addr"], xn["k_addr"], w.K, rows=rows)
    res = compare_indices(got_idx[:, rows], want_idx, xn["q_addr"], xn["k_addr"], rows=rows)
    assert not res["bad"], res["bad"][:5]
    want_out = oracle.sparse_meat_attention(xn["q"], xn["k"], xn["v"], got_idx[:, rows], w.D ** -0.5, rows=rows)
    assert np.abs(_np(out)[:, :, rows] - want_out).max() <= 2e-3
    _check_topk_properties(x["q_addr"], x["k_addr"], idx, w.K)


def _check_topk_properties(qa, ka, idx, K, block=2048):
    """Size-independent checks over every row: causal, unique, and no unretrieved key beats a retrieved one."""
    B, T, _ = qa.shape
    q = qa.float()
    k = ka.float()
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for b in range(B):
            for i0 in range(0, T, block):
                i1 = min(i0 + block, T)
                ii = idx[b, i0:i1].long()
                rows = torch.arange(i0, i1, device=qa.device)
                full = rows >= K - 1
                s = q[b, i0:i1] @ k[b, :i1].T
                s = s.masked_fill(torch.arange(i1, device=qa.device)[None] > rows[:, None], float("-inf"))
                sel = torch.gather(s, 1, ii.clamp(0, i1 - 1))
                assert (ii[full] <= rows[full, None]).all(), "non-causal index"
                srt = ii.sort(dim=1).values
                assert (srt[:, 1:] != srt[:, :-1])[full].all(), "duplicate index"
                s_rest = s.scatter(1, ii.clamp(0, i1 - 1), float("-inf"))
                min_sel = sel[full].min(dim=1).values
                max_rest = s_rest[full].max(dim=1).values
                slack = 1e-6 * min_sel.abs() + 1e-7
                assert (max_rest <= min_sel + slack).all(), "an unretrieved key scores above a retrieved one"

    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


@pytest.mark.parametrize("K", [1, 32, 64, 128, 256])
def test_clustered_near_ties_all_budgets(K, cuda_device):
    """cfg5's clustered addresses (near-tie stress) at reduced T, every K class, vs the oracle."""
    w = scaled(CONFIGS["cfg5"], B=2, H=2, T=1536, K=K)
    inp = make_inputs(w)
    x = to_device(inp, cuda_device)
    xn = {k: v.float().contiguous().numpy() for k, v in inp.items()}
    idx = causal_topk(x["q_addr"], x["k_addr"], K).cpu().numpy()
    want = oracle.causal_topk(xn["q_addr"], xn["k_addr"], K)
    res = compare_indices(idx, want, xn["q_addr"], xn["k_addr"])
    assert not res["bad"], res["bad"][:5]
    print(f"K={K}: {res['exempt']} near-tie rows of {res['rows']}")


@pytest.mark.parametrize("R", [8, 16, 32, 48, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_topk_address_dims_and_dtypes(R, dtype, cuda_device):
    K = 64 if R == 128 else 96
    w = Workload("t", 2, 1, 777, 16, R, K, dtype)
    inp = make_inputs(w)
    x = to_device(inp, cuda_device)
    xn = {k: v.float().contiguous().numpy() for k, v in inp.items()}
    got = causal_topk(x["q_addr"], x["k_addr"], K).cpu().numpy()
    want = oracle.causal_topk(xn["q_addr"], xn["k_addr"], K)
    res = compare_indices(got, want, xn["q_addr"], xn["k_addr"])
    assert not res["bad"], res["bad"][:5]
    assert same_selection(got[:, : K - 1], want[:, : K - 1])  # short rows: all their keys, pads exactly


@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 129, 200])
def test_topk_short_and_ragged_sequences(T, cuda_device):
    K = 128
    w = Workload("t", 3, 1, T, 16, 32, K, torch.float32)
    inp = make_inputs(w)
    x = to_device(inp, cuda_device)
    xn = {k: v.float().contiguous().numpy() for k, v in inp.items()}
    got = causal_topk(x["q_addr"], x["k_addr"], K).cpu().numpy()
    want = oracle.causal_topk(xn["q_addr"], xn["k_addr"], K)
    assert got.shape == (3, T, min(K, T))
    assert same_selection(got, want)


def test_topk_exact_ties_break_to_lower_index(cuda_device):
    """Duplicated key addresses give exactly equal scores; the lower index must win."""
    T, R, K = 512, 32, 16
    g = torch.Generator().manual_seed(3)
    base = torch.randn(8, R, generator=g)
    sel = torch.randint(0, 8, (1, T), generator=g)
    ka = base[sel]
    qa = torch.randn(1, T, R, generator=g)
    got = causal_topk(qa.to(cuda_device), ka.to(cuda_device), K).cpu().numpy()
    sel_np = sel[0].numpy()
    for i in range(K - 1, T):
        # score each distinct base vector once, so duplicated keys get bitwise-equal scores
        s = (base.double().numpy() @ qa[0, i].double().numpy())[sel_np[: i + 1]]
        want = np.lexsort((np.arange(i + 1), -s))[:K]
        assert sorted(got[0, i].tolist()) == sorted(want.tolist()), i


def test_topk_masked_pads(cuda_device):
    w = Workload("t", 1, 1, 300, 16, 32, 64, torch.float32)
    x = to_device(make_inputs(w), cuda_device)
    got = causal_topk(x["q_addr"], x["k_addr"], 64, pad_mode="masked").cpu().numpy()
    for i in range(63):
        assert (got[0, i, i + 1:] == -1).all()


def test_topk_row_map_sharding(cuda_device):
    """Cyclic query-row blocks (the long-sequence sharding) equal the same rows of a full call."""
    w = Workload("t", 1, 1, 4096, 16, 32, 128, torch.bfloat16)
    inp = make_inputs(w)
    x = to_device(inp, cuda_device)
    full = causal_topk(x["q_addr"], x["k_addr"], 128)
    from wayfinder_attention_b200.sharding import local_rows, sharded_causal_topk

    for world in (2, 4, 8):
        for rank in range(world):
            rows = local_rows(w.T, world, rank, tile=256)
            qa_local = x["q_addr"][:, torch.from_numpy(rows).to(cuda_device)]
            got = sharded_causal_topk(qa_local, x["k_addr"], 128, world, rank, tile=256)
            assert torch.equal(got, full[:, torch.from_numpy(rows).to(cuda_device)])


@pytest.mark.parametrize("D", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_attention_head_dims(D, dtype, cuda_device):
    w = Workload("t", 2, 3, 300, D, 32, 48, dtype)
    inp = make_inputs(w)
    x = to_device(inp, cuda_device)
    xn = {k: v.float().contiguous().numpy() for k, v in inp.items()}
    g = torch.Generator().manual_seed(11)
    idx = torch.randint(0, w.T, (w.B, w.T, w.K), generator=g, dtype=torch.int32)
    out = sparse_meat_attention(x["q"], x["k"], x["v"], idx.to(cuda_device), D ** -0.5, out_dtype=torch.float32)
    want = oracle.sparse_meat_attention(xn["q"], xn["k"], xn["v"], idx.numpy(), D ** -0.5)
    assert np.abs(_np(out) - want).max() <= 1e-5


def test_attention_index_semantics(cuda_device):
    """int64 indices are accepted, negatives wrap like torch indexing, or are masked on request."""
    w = Workload("t", 1, 2, 128, 64, 32, 8, torch.float32)
    inp = make_inputs(w)
    x = to_device(inp, cuda_device)
    xn = {k: v.float().contiguous().numpy() for k, v in inp.items()}
    g = torch.Generator().manual_seed(5)
    idx = torch.randint(-w.T, w.T, (1, w.T, w.K), generator=g)
    out = sparse_meat_attention(x["q"], x["k"], x["v"], idx.to(cuda_device), 0.125, out_dtype=torch.float32)
    want = oracle.sparse_meat_attention(xn["q"], xn["k"], xn["v"], idx.numpy(), 0.125)
    assert np.abs(_np(out) - want).max() <= 1e-5
    idx[..., 0] = idx[..., 0] % w.T  # keep one real key per row
    out = sparse_meat_attention(x["q"], x["k"], x["v"], idx.to(cuda_device), 0.125, out_dtype=torch.float32,
                                mask_negative=True)
    want = oracle.sparse_meat_attention(xn["q"], xn["k"], xn["v"], idx.numpy(), 0.125, mask_negative=True)
    assert np.abs(_np(out) - want).max() <= 1e-5


def test_attention_out_of_range_sets_status(cuda_device):
    w = Workload("t", 1, 2, 64, 64, 32, 4, torch.float32)
    x = to_device(make_inputs(w), cuda_device)
    idx = torch.zeros(1, 64, 4, dtype=torch.int32)
    idx[0, 5, 2] = 64  # out of range
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = sparse_meat_attention(x["q"], x["k"], x["v"], idx.to(cuda_device), 0.125, status=status)
    assert status.item() & 1
    assert torch.isnan(out[0, :, 5]).all()
    assert torch.isfinite(out[0, :, 6]).all()


def test_strided_views_need_no_copy(cuda_device):
    """BHTD views of BTHD memory (the module's layout) and contiguous BHTD give identical results."""
    w = Workload("t", 2, 4, 256, 64, 32, 32, torch.bfloat16)
    x = to_device(make_inputs(w), cuda_device)
    assert not x["q"].is_contiguous()
    a, ia = fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], 32, 0.125)
    b, ib = fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"].contiguous(), x["k"].contiguous(),
                                   x["v"].contiguous(), 32, 0.125)
    assert torch.equal(ia, ib) and torch.equal(a, b)


def test_errors_are_raised(cuda_device):
    w = Workload("t", 1, 2, 300, 64, 32, 8, torch.float32)
    x = to_device(make_inputs(w), cuda_device)
    with pytest.raises(ValueError):
        causal_topk(x["q_addr"], x["k_addr"], 257)  # beyond this build's maximum
    with pytest.raises(ValueError):
        causal_topk(x["q_addr"], x["k_addr"][:, :10], 8)
    with pytest.raises(RuntimeError):
        causal_topk(x["q_addr"].cpu(), x["k_addr"].cpu(), 8)
    assert causal_topk(x["q_addr"], x["k_addr"], 0).shape == (1, 300, 0)
    out, idx = fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], 0, 0.125)
    assert idx.shape == (1, 300, 0) and (out == 0).all()


def test_module_drop_in(cuda_device):
    """LearnedAddressSparseAttention: fused path equals projections + oracle composition."""
    from wayfinder_attention_b200 import LearnedAddressSparseAttention

    torch.manual_seed(45)
    m = LearnedAddressSparseAttention(128, 2, top_k=32, retrieval_config={"use_fused_sparse": True,
                                                                           "method": "fused_causal"}).eval()
    x = torch.randn(2, 200, 128)
    with torch.no_grad():
        q = m.q_proj(x).view(2, 200, 2, 64).transpose(1, 2)
        k = m.k_proj(x).view(2, 200, 2, 64).transpose(1, 2)
        v = m.v_proj(x).view(2, 200, 2, 64).transpose(1, 2)
        qa, ka = m.address.forward_query_key(x)
        o, _ = oracle.fused_sparse_attention(qa.numpy(), ka.numpy(), q.numpy(), k.numpy(), v.numpy(), 32, 64 ** -0.5)
        want = m.out_proj(torch.from_numpy(o).transpose(1, 2).reshape(2, 200, 128))
    m = m.to(cuda_device)
    got = m(x.to(cuda_device))
    assert (got.cpu() - want).abs().max() <= 1e-4
    got2, attn = m(x.to(cuda_device), return_attention=True)
    assert attn.shape == (2, 200, 200)
    assert torch.allclose(attn.sum(-1), torch.ones(2, 200, device=cuda_device))


def test_decoder_prefill_smoke(cuda_device):
    from wayfinder_attention_b200 import TransformerLM

    torch.manual_seed(45)
    m = TransformerLM(128, d_model=256, n_layers=2, n_heads=4, d_ff=1024, max_seq_len=512,
                      routing_top_k=128).to(cuda_device).eval()
    ids = torch.randint(0, 128, (2, 512), device=cuda_device)
    with torch.no_grad():
        logits = m(ids)["logits"]
    assert logits.shape == (2, 512, 128) and torch.isfinite(logits).all()


@pytest.mark.parametrize(
    "R,K,T,B,dtype,clustered",
    [
        (32, 128, 16384, 1, torch.bfloat16, False),
        (32, 128, 4096, 2, torch.bfloat16, True),
        (16, 64, 1000, 2, torch.float16, False),
        (64, 128, 3000, 1, torch.bfloat16, False),
        (32, 32, 777, 3, torch.bfloat16, True),
        (32, 1, 300, 1, torch.bfloat16, False),
        (32, 128, 130, 1, torch.bfloat16, False),
        (32, 256, 8192, 2, torch.bfloat16, True),   # K = 256: 384-slot lists, 8-register sort
        (64, 200, 2500, 1, torch.float16, False),
        (32, 256, 300, 1, torch.bfloat16, False),   # short rows: K_eff = 256 with pads
        (32, 128, 8192, 10, torch.bfloat16, True),  # 8 + 2 batch elements: two workspace slices
        (32, 128, 2048, 1, torch.float32, False),   # cfg1: fp32 addresses via bf16 copies + fp32 rescoring
        (16, 64, 3000, 2, torch.float32, True),
        (64, 256, 1500, 1, torch.float32, False),
    ],
)
def test_tensor_core_topk_equals_cuda_core(R, K, T, B, dtype, clustered, cuda_device, monkeypatch):
    """The tcgen05 scorer admits keys on tensor-core scores but ranks on exact fp32 rescoring,
    so it must select exactly the keys the CUDA-core kernel selects."""
    w = Workload("t", B, 1, T, 16, R, K, dtype, clustered=clustered)
    x = to_device(make_inputs(w), cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    tc = causal_topk(x["q_addr"], x["k_addr"], K, status=status)
    monkeypatch.setenv("WF_TOPK_IMPL", "cuda_core")
    cc = causal_topk(x["q_addr"], x["k_addr"], K)
    monkeypatch.delenv("WF_TOPK_IMPL")
    torch.cuda.synchronize()
    assert status.item() == 0
    # the same index set in every row (slot order is unspecified: the CUDA-core kernel
    # sorts by score, the tensor-core one keeps its lists' order); pads in the same slots
    mism = (tc.sort(dim=-1).values != cc.sort(dim=-1).values).any(dim=-1)
    assert not mism.any(), f"{int(mism.sum())} rows differ, first {torch.nonzero(mism)[:5].tolist()}"
    T_ = x["q_addr"].shape[1]
    k_eff = min(K, T_)
    for i in range(min(k_eff - 1, T_)):
        assert torch.equal(tc[:, i, i + 1:], cc[:, i, i + 1:])


def test_workspace_too_small_is_rejected(cuda_device):
    import ctypes

    from wayfinder_attention_b200 import _lib

    w = Workload("t", 1, 1, 512, 16, 32, 64, torch.bfloat16)
    x = to_device(make_inputs(w), cuda_device)
    lib = _lib.load_library()
    idx = torch.empty(1, 512, 64, dtype=torch.int32, device=cuda_device)
    ws = torch.empty(1024, dtype=torch.uint8, device=cuda_device)
    rc = lib.wf_causal_topk(x["q_addr"].data_ptr(), x["k_addr"].data_ptr(), _lib.WF_DTYPE_BF16, 1, 512, 512, 32,
                            _lib.strides(x["q_addr"]), _lib.strides(x["k_addr"]), 64, 0, 0, 1, 0, idx.data_ptr(),
                            ws.data_ptr(), ws.numel(), None, _lib.stream_ptr(cuda_device))
    assert rc == _lib.WF_ERR_INVALID_ARGUMENT and b"workspace" in lib.wf_last_error()


@pytest.mark.parametrize("fused", [True, False])
def test_key_vector_module_matches_oracle(fused, cuda_device):
    """KeyVectorSparseAttention: head-mean search vectors (R = head_dim = 64) through the same kernels."""
    from wayfinder_attention_b200 import KeyVectorSparseAttention

    torch.manual_seed(45)
    m = KeyVectorSparseAttention(256, 4, top_k=64, retrieval_config={"use_fused_sparse": fused}).eval()
    x = torch.randn(2, 300, 256)
    with torch.no_grad():
        q = m.q_proj(x).view(2, 300, 4, 64).transpose(1, 2)
        k = m.k_proj(x).view(2, 300, 4, 64).transpose(1, 2)
        v = m.v_proj(x).view(2, 300, 4, 64).transpose(1, 2)
        qs, ks = k.mean(dim=1), q.mean(dim=1)  # the reference's argument order
        o, _ = oracle.fused_sparse_attention(qs.numpy(), ks.numpy(), q.numpy(), k.numpy(), v.numpy(), 64, 0.125)
        want = m.out_proj(torch.from_numpy(o).transpose(1, 2).reshape(2, 300, 256))
    got = m.to(cuda_device)(x.to(cuda_device))
    assert (got.cpu() - want).abs().max() <= 1e-4
