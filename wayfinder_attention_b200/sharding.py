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


def _all_gather_rows(x_local: torch.Tensor, world: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather (B, Tl, ...) shards along dim 1 into a rank-major (world, B, Tl, ...) tensor."""
    import torch.distributed as dist

    x_local = x_local.contiguous()
    shape = (world,) + tuple(x_local.shape)
    if out is None or tuple(out.shape) != shape or out.dtype != x_local.dtype or out.device != x_local.device:
        out = torch.empty(shape, dtype=x_local.dtype, device=x_local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, x_local, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), x_local, group=group)
    return out


def gather_sequence(x_local: torch.Tensor, tile: int, group=None) -> torch.Tensor:
    """Rebuild the full sequence from cyclic row-block shards.

    x_local: (B, Tl, ...) holding this rank's rows ``local_rows(T, world, rank, tile)`` in order.
    Returns (B, T, ...) in global row order.  Requires T = world * Tl with Tl a multiple of
    ``tile`` (every rank holds the same number of whole blocks).  One all-gather
    (NCCL over NVLink on GPUs, any backend elsewhere) plus one reordering copy.
    """
    import torch.distributed as dist

    B, Tl = x_local.shape[0], x_local.shape[1]
    if Tl % tile:
        raise ValueError(f"local rows {Tl} are not a whole number of {tile}-row blocks")
    world = dist.get_world_size(group)
    g = _all_gather_rows(x_local, world, group)  # (W, B, Tl, ...)
    nblk = Tl // tile
    rest = tuple(x_local.shape[2:])
    g = g.view((world, B, nblk, tile) + rest)
    # global block index = local block * world + rank
    g = g.permute((1, 2, 0, 3) + tuple(range(4, 4 + len(rest))))
    return g.reshape((B, world * Tl) + rest)


class SequenceShardedAttention:
    """Fused retrieval + sparse attention for ONE long sequence split over ranks.

    Rank r holds the query rows ``local_rows(T, W, r, tile)`` of the addresses and of
    q/k/v (in the module's (B, T, H, D) memory layout).  Every rank needs all key
    addresses and every K/V row up to its last query, so ``forward``:
      1. all-gathers the key addresses (B*T*d_A elements, small) and starts the
         K/V all-gather on a side stream;
      2. runs the causal top-K of its own rows against all keys (row map of
         ``wf_causal_topk``) while K/V are in flight;
      3. waits for K/V and runs the sparse attention of its rows.
    The K/V all-gathers land rank-major and the attention kernel translates key
    positions to (rank, local row) itself, so no reordering copy of K/V is made.
    The only collectives are these all-gathers; nothing crosses ranks afterwards.
    """

    def __init__(self, top_k: int, scale: float, tile: int = 256, group=None, pad_mode: str = "reference"):
        self.top_k = top_k
        self.scale = scale
        self.tile = tile
        self.group = group
        self.pad_mode = pad_mode
        # persistent per-shape gather buffers and side stream: a forward allocates nothing large
        self._kg = None
        self._vg = None
        self._side = None

    def forward(self, q_addr_l: torch.Tensor, k_addr_l: torch.Tensor, q_l: torch.Tensor, k_l: torch.Tensor,
                v_l: torch.Tensor, out_dtype: torch.dtype | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """q_addr_l, k_addr_l: (B, Tl, R); q_l, k_l, v_l: (B, H, Tl, D) views of (B, Tl, H, D) memory."""
        import torch.distributed as dist

        from . import _lib

        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        B, H, Tl, D = q_l.shape
        T = world * Tl
        main = torch.cuda.current_stream(q_l.device)
        if self._side is None or self._side.device != q_l.device:
            self._side = torch.cuda.Stream(device=q_l.device)
        side = self._side
        side.wait_stream(main)  # the previous call's attention has finished with the buffers
        with torch.cuda.stream(side):
            # rank-major (world, B, Tl, H, D): the attention kernel addresses it directly
            self._kg = k_g = _all_gather_rows(k_l.transpose(1, 2), world, self.group, self._kg)
            self._vg = v_g = _all_gather_rows(v_l.transpose(1, 2), world, self.group, self._vg)
        k_addr = gather_sequence(k_addr_l, self.tile, self.group)  # small: reordered to global order
        idx = sharded_causal_topk(q_addr_l, k_addr, self.top_k, world, rank, self.tile, self.pad_mode)
        main.wait_stream(side)
        dev = q_l.device
        out = torch.empty(B, H, Tl, D, dtype=out_dtype or q_l.dtype, device=dev)
        kb = k_g[0].transpose(1, 2)  # rank 0's block as (B, H, Tl, D)
        vb = v_g[0].transpose(1, 2)
        K = idx.shape[-1]
        lib = _lib.load_library()
        with torch.cuda.device(dev):
            rc = lib.wf_sparse_attention_cyclic_kv(
                q_l.data_ptr(), kb.data_ptr(), vb.data_ptr(), _lib.dtype_code(q_l.dtype), idx.data_ptr(),
                B, H, Tl, T, D, K, _lib.strides(q_l), _lib.strides(kb), _lib.strides(vb), _lib.strides(idx),
                float(self.scale), _lib.WF_ATTN_MASK_NEGATIVE if self.pad_mode == "masked" else 0,
                out.data_ptr(), _lib.dtype_code(out.dtype), _lib.strides(out), self.tile, world,
                k_g.stride(0), v_g.stride(0), None, _lib.stream_ptr(dev),
            )
        _lib.check(rc)
        return out, idx

    __call__ = forward
