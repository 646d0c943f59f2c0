"""Work partitioning of the hot path over the GPUs of one node.

The reference is single-GPU only; these plans come from the forward's own
independence structure:
  * retrieval is independent per batch element and attention per
    (batch element, head), so a batch (or batch x head) split needs no
    collective at all (``batch_shard``);
  * one long sequence is split by query-row blocks assigned cyclically
    (``local_rows``): rank r owns global blocks r, r + W, r + 2W, ... of
    ``tile`` rows, which balances the causal triangle.  Each rank then needs
    every key address and every K/V row up to its last query, which it gets
    by all-gathering the small per-rank shards (``SequenceShardedAttention``).
"""

from __future__ import annotations

import numpy as np
import torch

from .causal_topk import _launch_topk, promote_compute_dtype


def batch_shard(B: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) batch range of ``rank``; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(B, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def local_rows(T: int, world: int, rank: int, tile: int) -> np.ndarray:
    """Global sequence positions owned by ``rank`` under cyclic query-row blocks of ``tile`` rows."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if tile < 64 or tile % 64:
        raise ValueError(f"tile must be a positive multiple of 64, got {tile}")
    nblk = (T + tile - 1) // tile
    blocks = np.arange(rank, nblk, world)
    if blocks.size == 0:
        return np.zeros(0, dtype=np.int64)
    rows = (blocks[:, None] * tile + np.arange(tile)[None, :]).reshape(-1)
    return rows[rows < T]


def sharded_causal_topk(q_addr_local: torch.Tensor, k_addr_full: torch.Tensor, top_k: int, world: int,
                        rank: int, tile: int, pad_mode: str = "reference") -> torch.Tensor:
    """Causal top-K for this rank's query rows (``local_rows`` order) against all keys.

    q_addr_local: (B, Tl, R) rows ``local_rows(T, world, rank, tile)``; k_addr_full: (B, T, R).
    Returns (B, Tl, min(top_k, T)) int32 with global key indices.
    """
    if q_addr_local.dim() != 3 or k_addr_full.dim() != 3 or q_addr_local.shape[::2] != k_addr_full.shape[::2]:
        raise ValueError(f"expected (B,Tl,R) and (B,T,R), got {tuple(q_addr_local.shape)}, {tuple(k_addr_full.shape)}")
    T = k_addr_full.shape[1]
    expect = local_rows(T, world, rank, tile).size
    if q_addr_local.shape[1] != expect:
        raise ValueError(f"rank {rank} of {world} owns {expect} rows at tile={tile}, got {q_addr_local.shape[1]}")
    q, k, _ = promote_compute_dtype(q_addr_local, k_addr_full)
    return _launch_topk(q, k, top_k, pad_mode, row_tile=tile, row_stride=world, row_start=rank)
