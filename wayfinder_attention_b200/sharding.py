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


def chunked_kv_attention(q_l: torch.Tensor, idx: torch.Tensor, k_g: torch.Tensor, v_g: torch.Tensor, scale: float,
                         tile: int, pad_mode: str = "reference", out_dtype: torch.dtype | None = None,
                         wait=None) -> torch.Tensor:
    """Attention of a rank's query rows over all-gathered K/V stored chunk-major.

    q_l: (B, H, Tl, D) this rank's rows (``local_rows`` order); idx: (B, Tl, K) global
    key indices; k_g, v_g: (C, W, B, Tc, H, D) with block (c, w) = rank w's local rows
    [c*Tc, (c+1)*Tc).  Chunk c of the query rows reads key chunks <= c only (causal),
    so chunks run in the order 1..C-1, 0 (chunk 0 last: the reference pads of rows
    t < K-1 point ahead) and ``wait(c)``, if given, is called before chunk c is
    enqueued — the caller makes the stream wait for that chunk's K/V there.
    """
    from . import _lib

    C, W, B, Tc, H, D = k_g.shape
    Tl = q_l.shape[2]
    if Tl != C * Tc or tuple(v_g.shape) != tuple(k_g.shape) or q_l.shape[0] != B or q_l.shape[1] != H:
        raise ValueError(f"q {tuple(q_l.shape)} does not match chunk-major K/V {tuple(k_g.shape)}")
    T = W * Tl
    dev = q_l.device
    out = torch.empty(B, H, Tl, D, dtype=out_dtype or q_l.dtype, device=dev)
    kb = k_g[0, 0].permute(0, 2, 1, 3)  # block (chunk 0, rank 0) as (B, H, Tc, D)
    vb = v_g[0, 0].permute(0, 2, 1, 3)
    K = idx.shape[-1]
    lib = _lib.load_library()
    flags = _lib.WF_ATTN_MASK_NEGATIVE if pad_mode == "masked" else 0
    st = _lib.status_arg(dev, None)
    with torch.cuda.device(dev):
        for c in list(range(1, C)) + [0]:
            if wait is not None:
                wait(c)
            rows = slice(c * Tc, (c + 1) * Tc)
            qc, ic, oc = q_l[:, :, rows], idx[:, rows], out[:, :, rows]
            rc = lib.wf_sparse_attention_cyclic_kv_chunked(
                qc.data_ptr(), kb.data_ptr(), vb.data_ptr(), _lib.dtype_code(q_l.dtype), ic.data_ptr(),
                B, H, Tc, T, D, K, _lib.strides(qc), _lib.strides(kb), _lib.strides(vb), _lib.strides(ic),
                float(scale), flags, oc.data_ptr(), _lib.dtype_code(out.dtype), _lib.strides(oc),
                tile, W, Tc, k_g.stride(1), v_g.stride(1), st, _lib.stream_ptr(dev),
            )
            _lib.check(rc)
    _lib.status_after(dev, None)
    return out


class SequenceShardedAttention:
    """Fused retrieval + sparse attention for ONE long sequence split over ranks.

    Rank r holds the query rows ``local_rows(T, W, r, tile)`` of the addresses and of
    q/k/v (in the module's (B, T, H, D) memory layout).  Every rank needs all key
    addresses and every K/V row up to its last query, so ``forward``:
      1. all-gathers the key addresses (B*T*d_A elements, small) and, on a side
         stream, the K/V rows in ``chunks`` chunks of local rows;
      2. runs the causal top-K of its own rows against all keys (row map of
         ``wf_causal_topk``) while K/V are in flight;
      3. runs the attention of its rows chunk by chunk as the K/V chunks land: the
         indices are causal, so local rows in chunk c read keys from chunks <= c of
         every rank.  Chunk 0 goes last because the reference pads of rows t < K-1
         (all in chunk 0 of rank 0, tile >= K) point at later keys.
    The K/V all-gathers land chunk-major and the attention kernel maps key positions
    to (chunk, rank, row) itself (``wf_sparse_attention_cyclic_kv_chunked``), so no
    reordering copy of K/V is made.  The only collectives are these all-gathers.
    """

    def __init__(self, top_k: int, scale: float, tile: int = 256, group=None, pad_mode: str = "reference",
                 chunks: int | None = None):
        self.top_k = top_k
        self.scale = scale
        self.tile = tile
        self.group = group
        self.pad_mode = pad_mode
        self.chunks = chunks
        # persistent per-shape gather buffers and side stream: a forward allocates nothing large
        self._kg = None
        self._vg = None
        self._side = None

    def _n_chunks(self, Tl: int, world: int) -> int:
        # Default: one chunk on 2 ranks, where retrieval already hides the gather
        # (cfg4: 9.38 ms unchunked, 9.55 ms in 8 chunks), 8 chunks from 4 ranks up,
        # where each rank receives (W-1)/W of K/V while its retrieval shrinks as 1/W.
        want = self.chunks if self.chunks is not None else (1 if world <= 2 else 8)
        c = max(1, min(want, 64 // world, Tl // self.tile))
        while c > 1 and Tl % (c * self.tile):
            c -= 1
        return c

    def forward(self, q_addr_l: torch.Tensor, k_addr_l: torch.Tensor, q_l: torch.Tensor, k_l: torch.Tensor,
                v_l: torch.Tensor, out_dtype: torch.dtype | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """q_addr_l, k_addr_l: (B, Tl, R); q_l, k_l, v_l: (B, H, Tl, D) views of (B, Tl, H, D) memory."""
        import torch.distributed as dist

        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        B, H, Tl, D = q_l.shape
        if self.top_k > self.tile:
            raise ValueError(f"top_k={self.top_k} must not exceed the row tile {self.tile}")
        C = self._n_chunks(Tl, world)
        Tc = Tl // C
        main = torch.cuda.current_stream(q_l.device)
        if self._side is None or self._side.device != q_l.device:
            self._side = torch.cuda.Stream(device=q_l.device)
        side = self._side
        shape = (C, world, B, Tc, H, D)
        kt, vt = k_l.transpose(1, 2), v_l.transpose(1, 2)  # (B, Tl, H, D)
        if self._kg is None or tuple(self._kg.shape) != shape or self._kg.dtype != k_l.dtype or self._kg.device != k_l.device:
            self._kg = torch.empty(shape, dtype=k_l.dtype, device=k_l.device)
            self._vg = torch.empty(shape, dtype=v_l.dtype, device=v_l.device)
        k_g, v_g = self._kg, self._vg
        # The key addresses (small) go first: collectives of one process group run in
        # issue order, so issued after the K/V chunks the retrieval would wait for them.
        k_addr = gather_sequence(k_addr_l, self.tile, self.group)  # reordered to global order
        side.wait_stream(main)  # the previous call's attention has finished with the buffers
        landed = []
        with torch.cuda.stream(side):
            for c in range(C):
                rows = slice(c * Tc, (c + 1) * Tc)
                _all_gather_rows(kt[:, rows], world, self.group, k_g[c])
                _all_gather_rows(vt[:, rows], world, self.group, v_g[c])
                ev = torch.cuda.Event()
                ev.record(side)
                landed.append(ev)
        idx = sharded_causal_topk(q_addr_l, k_addr, self.top_k, world, rank, self.tile, self.pad_mode)
        out = chunked_kv_attention(q_l, idx, k_g, v_g, self.scale, self.tile, self.pad_mode, out_dtype,
                                   wait=lambda c: main.wait_event(landed[c] if c else landed[-1]))
        return out, idx

    __call__ = forward
