"""CPU oracle for the Wayfinder hot path — TEST INFRASTRUCTURE, NOT THE PRODUCT.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker or the timed CPU
baseline.  The product (``wayfinder_attention_b200``) never calls it.

It restates, in numpy fp32, the reference's own PyTorch path for
``fused_sparse_attention(..., retrieval_method="fused_causal")`` on CPU:

  causal_topk            <- routing_attention/kernels/causal_topk.py:470-521
    row blocks           <- _pick_row_block                       causal_topk.py:75-83
    fp32 block scores    <- _causal_topk_row_blocked bmm          causal_topk.py:150-160
    causal mask          <- _apply_causal_mask_scores             causal_topk.py:110-129
    top-K per row        <- torch.topk(k_eff)                      causal_topk.py:167
    pads for short rows  <- _finalize_causal_topk                 causal_topk.py:37-57
  sparse_meat_attention  <- sparse_meat_attention_reference      fused_sparse.py:80-94
    gather               <- _gather_kv_batched                    fused_sparse.py:64-77

Two choices the reference leaves open are fixed here: ties at the K-th score
break to the lower key index (as in the CUDA kernels), slots are sorted by
descending score (the reference's ``topk(sorted=False)`` order is
implementation-defined, and so is the CUDA kernels' — comparisons are by index
set), and the pad slots of rows i < K-1 are the trailing slots s = i+1 .. K-1
(the reference pads whichever slots topk left at -inf; the CUDA kernels use the
trailing slots too).

Parity pin: ``tests/golden/`` holds outputs of the reference itself, produced
by ``tests/golden/make_golden.py`` importing the reference in the build
container; ``tests/test_oracle_golden.py`` checks this module against them.
"""

from __future__ import annotations

import numpy as np


def pick_row_block(T: int) -> int:
    """Row-block size of ``_pick_row_block`` (causal_topk.py:75-83)."""
    if T >= 16384:
        return 4096
    if T >= 8192:
        return 2048
    if T >= 2048:
        return 1024
    return 512


def _select_block(s: np.ndarray, rows: np.ndarray, K: int, T: int, pad_mode: str) -> np.ndarray:
    """Exact top-K of each row of ``s`` (already -inf beyond the causal limit).

    Returns (nrows, K) int32: valid slots sorted by (score desc, index asc), then pads.
    """
    n_rows, n_cols = s.shape
    out = np.empty((n_rows, K), dtype=np.int32)
    n_valid = np.minimum(rows + 1, K)
    if n_cols > K:
        kth = -np.partition(-s, K - 1, axis=1)[:, K - 1]
    else:
        kth = np.full(n_rows, -np.inf, dtype=s.dtype)
    for r in range(n_rows):
        row = s[r]
        n = int(n_valid[r])
        if n < K or n_cols <= K:
            cand = np.arange(min(int(rows[r]) + 1, n_cols))
        else:
            t = kth[r]
            gt = np.nonzero(row > t)[0]
            eq = np.nonzero(row == t)[0][: K - gt.size]  # lowest indices among the tie
            cand = np.concatenate([gt, eq])
        order = np.lexsort((cand, -row[cand].astype(np.float64)))
        sel = cand[order][:n]
        out[r, :n] = sel
        if n < K:
            slots = np.arange(n, K)
            out[r, n:] = (rows[r] + K + slots + 1) % T if pad_mode == "reference" else -1
    return out


def causal_topk(q: np.ndarray, k: np.ndarray, top_k: int, *, pad_mode: str = "reference",
                rows: np.ndarray | None = None) -> np.ndarray:
    """(B,T,R) x (B,T,R) float -> (B, n_rows, min(top_k, T)) int32 exact causal top-K.

    ``rows`` optionally restricts the query rows (default: all T rows).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    if q.shape != k.shape or q.ndim != 3:
        raise ValueError(f"expected matching (B,T,R) inputs, got {q.shape} and {k.shape}")
    B, T, _ = q.shape
    K = min(int(top_k), T)
    rows = np.arange(T) if rows is None else np.asarray(rows, dtype=np.int64)
    out = np.empty((B, rows.size, max(K, 0)), dtype=np.int32)
    if K == 0 or rows.size == 0:
        return out
    bm = pick_row_block(T)
    for b in range(B):
        for a in range(0, rows.size, bm):
            rr = rows[a:a + bm]
            i1 = int(rr.max()) + 1
            s = q[b, rr] @ k[b, :i1].T  # fp32, like the bmm at causal_topk.py:160
            s[np.arange(i1)[None, :] > rr[:, None]] = -np.inf
            out[b, a:a + rr.size] = _select_block(s, rr, K, T, pad_mode)
    return out


def causal_topk_key_mask(q: np.ndarray, k: np.ndarray, top_k: int, key_mask: np.ndarray) -> np.ndarray:
    """Causal top-K over the keys a (B, T) padding mask keeps; unfilled slots are -1.

    The reference's sparse path ignores its attn_mask (models/attention.py:456-490);
    the semantics here are those of its dense path, which drops masked keys
    (attention.py:157-167, mask built as input_ids != pad at transformer.py:269-270):
    query t ranks keys j <= t with key_mask[b, j] != 0 by fp32 score, ties to the
    lower index.  Small cases only (a Python loop over rows).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    B, T, _ = q.shape
    K = min(int(top_k), T)
    out = np.full((B, T, K), -1, dtype=np.int32)
    for b in range(B):
        valid = np.nonzero(np.asarray(key_mask[b]) != 0)[0]
        for t in range(T):
            cand = valid[valid <= t]
            if cand.size == 0:
                continue
            sc = (k[b, cand] @ q[b, t]).astype(np.float32)
            order = np.lexsort((cand, -sc.astype(np.float64)))
            sel = cand[order][:K]
            out[b, t, : sel.size] = sel
    return out


def sparse_meat_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, idx: np.ndarray, scale: float, *,
                          mask_negative: bool = False, rows: np.ndarray | None = None,
                          chunk: int = 256) -> np.ndarray:
    """fp32 gather + softmax + weighted sum (``sparse_meat_attention_reference``, fused_sparse.py:80-94).

    q: (B,H,Tq,D); k, v: (B,H,Tk,D); idx: (B,Tq,K).  ``rows`` restricts the query rows
    (idx then holds only those rows).  Negative indices wrap like numpy/torch indexing
    unless ``mask_negative``.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    B, H, Tq, D = q.shape
    rows = np.arange(Tq) if rows is None else np.asarray(rows, dtype=np.int64)
    Kn = idx.shape[-1]
    out = np.zeros((B, H, rows.size, D), dtype=np.float32)
    if Kn == 0:
        return out
    for b in range(B):
        for a in range(0, rows.size, chunk):
            rr = rows[a:a + chunk]
            ii = np.asarray(idx[b, a:a + rr.size], dtype=np.int64)  # (n, K)
            masked = ii < 0 if mask_negative else np.zeros(ii.shape, dtype=bool)
            jj = np.where(masked, 0, ii)
            ks = k[b][:, jj]  # (H, n, K, D)
            vs = v[b][:, jj]
            qq = q[b][:, rr]  # (H, n, D)
            s = np.einsum("hnd,hnkd->hnk", qq, ks, dtype=np.float32) * np.float32(scale)
            s = np.where(masked[None], -np.inf, s)
            m = s.max(axis=-1, keepdims=True)
            e = np.exp(s - m)
            p = e / e.sum(axis=-1, keepdims=True)
            out[b, :, a:a + rr.size] = np.einsum("hnk,hnkd->hnd", p, vs, dtype=np.float32)
    return out


def fused_sparse_attention(q_addr, k_addr, q, k, v, top_k: int, scale: float, *, pad_mode: str = "reference",
                           rows: np.ndarray | None = None):
    """Retrieval then attention (fused_sparse.py:327-356).  Returns (out, idx)."""
    idx = causal_topk(q_addr, k_addr, top_k, pad_mode=pad_mode, rows=rows)
    out = sparse_meat_attention(q, k, v, idx, scale, mask_negative=pad_mode == "masked", rows=rows)
    return out, idx


def exact_scores_f64(q_addr: np.ndarray, k_addr: np.ndarray, b: int, i: int) -> np.ndarray:
    """fp64 scores of query row i against keys 0..i (used for the near-tie exemption)."""
    return k_addr[b, : i + 1].astype(np.float64) @ q_addr[b, i].astype(np.float64)
