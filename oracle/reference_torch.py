"""The reference's CPU path restated with the same PyTorch operations — TEST AND
BASELINE INFRASTRUCTURE, NOT THE PRODUCT.

Only ``tests/`` and ``bench.py``'s CPU-baseline / reference arm may import this
module.  Where ``wayfinder_oracle`` restates the reference's arithmetic in numpy
(the parity checker), this module restates its *execution*: the same torch CPU
operations in the same order and shapes, so that timing it on the host cores
measures what the reference's own fp32 CPU path costs
(``fused_sparse_attention(..., retrieval_method="fused_causal")`` on CPU):

  row-blocked causal top-K  <- routing_attention/kernels/causal_topk.py:133-171
    fp32 upcast, bmm of a row block against its causal key prefix   :150-160
    keys beyond each row masked to -inf                             :111-129, :161-165
    topk(k_eff, sorted=False) per row                               :167
    pad index (row + k_eff + slot + 1) % T for -inf slots           :37-57
  gather attention          <- routing_attention/kernels/fused_sparse.py:64-94
    k_sel / v_sel of shape (B, H, n, K, D) by advanced indexing     :64-77
    scores = q @ k_sel^T * scale, softmax, (p * v_sel).sum         :80-94

``rows`` restricts the query rows (the bounded sample of the timed baseline): each
block of sampled rows is scored against the key prefix its last row can see, as a
row block of the reference is.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def row_block(T: int) -> int:
    """Rows per block, as ``_pick_row_block`` chooses them (causal_topk.py:76-83)."""
    return 4096 if T >= 16384 else 2048 if T >= 8192 else 1024 if T >= 2048 else 512


@torch.no_grad()
def causal_topk(q_addr: torch.Tensor, k_addr: torch.Tensor, top_k: int,
                rows: torch.Tensor | None = None) -> torch.Tensor:
    """(B, T, R) x (B, T, R) -> (B, n, k_eff) int32 for the query rows ``rows`` (default: all)."""
    B, T, _ = q_addr.shape
    k_eff = min(top_k, T)
    q = q_addr.float()
    k = k_addr.float()
    rows = torch.arange(T) if rows is None else rows.long()
    out = torch.empty(B, rows.numel(), k_eff, dtype=torch.int32)
    bm = row_block(T)
    for a in range(0, rows.numel(), bm):
        rr = rows[a:a + bm]
        n_keys = int(rr.max()) + 1
        scores = torch.bmm(q[:, rr], k[:, :n_keys].transpose(1, 2).contiguous())
        future = torch.arange(n_keys).view(1, n_keys) > rr.view(-1, 1)
        scores = scores.masked_fill(future.unsqueeze(0), float("-inf"))
        if n_keys < k_eff:  # fewer keys than slots: every slot past them is a pad
            scores = F.pad(scores, (0, k_eff - n_keys), value=float("-inf"))
        vals, idx = torch.topk(scores, k=k_eff, dim=-1, sorted=False)
        slots = torch.arange(k_eff).view(1, 1, k_eff)
        pad = (rr.view(1, -1, 1) + k_eff + slots + 1) % T
        valid = vals.isfinite() & (vals > -1e30)
        out[:, a:a + rr.numel()] = torch.where(valid, idx, pad).to(torch.int32)
    return out


@torch.no_grad()
def sparse_meat_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, idx: torch.Tensor,
                          scale: float) -> torch.Tensor:
    """q: (B, H, n, D) query rows; k, v: (B, H, T, D); idx: (B, n, K) -> (B, H, n, D) fp32."""
    q, k, v = q.float(), k.float(), v.float()
    B, H = k.shape[0], k.shape[1]
    bi = torch.arange(B).view(B, 1, 1, 1)
    hi = torch.arange(H).view(1, H, 1, 1)
    sel = idx.long().unsqueeze(1)
    k_sel = k[bi, hi, sel, :]
    v_sel = v[bi, hi, sel, :]
    scores = torch.matmul(q.unsqueeze(-2), k_sel.transpose(-2, -1)).squeeze(-2) * scale
    p = F.softmax(scores, dim=-1)
    return (p.unsqueeze(-1) * v_sel).sum(dim=-2)


@torch.no_grad()
def fused_sparse_attention(q_addr, k_addr, q, k, v, top_k: int, scale: float, rows: torch.Tensor | None = None):
    """Retrieval then attention for the query rows ``rows``: (out (B, H, n, D), idx (B, n, K))."""
    T = q_addr.shape[1]
    rows = torch.arange(T) if rows is None else rows.long()
    idx = causal_topk(q_addr, k_addr, top_k, rows)
    out = sparse_meat_attention(q[:, :, rows], k, v, idx, scale)
    return out, idx
