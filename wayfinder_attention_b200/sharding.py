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
    so chunks run in order and ``wait(c, everything)``, if given, is called before
    chunk c is enqueued — the caller makes the stream wait there for key chunks
    0..c, or for all of them when ``everything`` is set.  That is the case for chunk
    0 when the reference pads of rows t < K-1 (global rows up to 3K-2) may lie
    beyond key chunk 0 (3K-2 >= Tc*W); chunk 0 then runs last.
    """
    C, W, B, Tc, H, D = k_g.shape
    if tuple(v_g.shape) != tuple(k_g.shape) or not k_g.is_contiguous() or not v_g.is_contiguous():
        raise ValueError(f"k_g / v_g must be contiguous chunk-major (C, W, B, Tc, H, D), got {tuple(k_g.shape)}")
    return _chunked_attention(q_l, idx, k_g.data_ptr(), v_g.data_ptr(), (C, W, B, Tc, H, D), scale, tile, pad_mode,
                              out_dtype, wait)


def _chunked_attention(q_l, idx, k_base: int, v_base: int, shape, scale, tile, pad_mode, out_dtype, wait):
    """``chunked_kv_attention`` on raw device addresses of contiguous (C, W, B, Tc, H, D) K/V buffers."""
    import ctypes

    from . import _lib

    C, W, B, Tc, H, D = shape
    Tl = q_l.shape[2]
    if Tl != C * Tc or q_l.shape[0] != B or q_l.shape[1] != H or q_l.shape[3] != D:
        raise ValueError(f"q {tuple(q_l.shape)} does not match chunk-major K/V {tuple(shape)}")
    T = W * Tl
    dev = q_l.device
    out = torch.empty(B, H, Tl, D, dtype=out_dtype or q_l.dtype, device=dev)
    # block (chunk 0, rank 0) as a (B, H, Tc, D) view of (B, Tc, H, D) memory
    kv_strides = (ctypes.c_int64 * 4)(Tc * H * D, D, H * D, 1)
    block = B * Tc * H * D
    K = idx.shape[-1]
    lib = _lib.load_library()
    flags = _lib.WF_ATTN_MASK_NEGATIVE if pad_mode == "masked" else 0
    st = _lib.status_arg(dev, None)
    zero_last = 3 * K - 2 >= Tc * W
    order = list(range(1, C)) + [0] if zero_last else list(range(C))
    with torch.cuda.device(dev):
        for c in order:
            if wait is not None:
                wait(c, c == 0 and zero_last)
            rows = slice(c * Tc, (c + 1) * Tc)
            qc, ic, oc = q_l[:, :, rows], idx[:, rows], out[:, :, rows]
            rc = lib.wf_sparse_attention_cyclic_kv_chunked(
                qc.data_ptr(), k_base, v_base, _lib.dtype_code(q_l.dtype), ic.data_ptr(),
                B, H, Tc, T, D, K, _lib.strides(qc), kv_strides, kv_strides, _lib.strides(ic),
                float(scale), flags, oc.data_ptr(), _lib.dtype_code(out.dtype), _lib.strides(oc),
                tile, W, Tc, block, block, st, _lib.stream_ptr(dev),
            )
            _lib.check(rc)
    _lib.status_after(dev, None)
    return out


class _PeerKV:
    """Chunk-major K/V gather buffer shared through CUDA IPC, filled by copy-engine pulls.

    Layout (2, C, W, B, Tc, H, D): tensor 0 is K, 1 is V; block (c, w) holds rank w's
    local rows [c*Tc, (c+1)*Tc).  Every rank packs its own blocks, then pulls the
    other ranks' blocks straight from their buffers over NVLink (``wf_peer_pull_blocks``).
    Two one-element all-reduces order the exchange across ranks: before packing
    (every peer has finished pulling the previous call's blocks) and before pulling
    (every peer has packed this call's).
    """

    def __init__(self, shape, dtype: torch.dtype, dev: torch.device, group, n_streams: int = 1):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self.shape = tuple(shape)
        self.dtype = dtype
        self.dev = dev
        self.group = group
        C, W, B, Tc, H, D = self.shape
        self.esz = torch.empty((), dtype=dtype).element_size()
        self.block = B * Tc * H * D * self.esz
        self.nbytes = 2 * C * W * self.block
        lib = _lib.load_library()
        self.lib = lib
        self.rank = dist.get_rank(group)
        self.world = W
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(dev):
            _lib.check(lib.wf_peer_buffer_alloc(self.nbytes, ctypes.byref(ptr), handle))
        self.own = ptr.value
        handles = [None] * W
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases = (ctypes.c_void_p * W)()
        self.opened = []
        with torch.cuda.device(dev):
            for p in range(W):
                if p == self.rank:
                    self.bases[p] = self.own
                    continue
                hp = (ctypes.c_uint8 * 64).from_buffer_copy(handles[p])
                peer = ctypes.c_void_p()
                _lib.check(lib.wf_peer_buffer_open(hp, ctypes.byref(peer)))
                self.bases[p] = peer.value
                self.opened.append(peer.value)
        self.streams = [torch.cuda.Stream(device=dev) for _ in range(max(1, min(n_streams, C)))]
        self.stream_ptrs = (ctypes.c_void_p * len(self.streams))(*[s.cuda_stream for s in self.streams])
        self.events = [torch.cuda.Event() for _ in range(C)]
        cur = torch.cuda.current_stream(dev)
        for e in self.events:  # create the CUDA events (torch creates them at the first record)
            e.record(cur)
        self.event_ptrs = (ctypes.c_void_p * C)(*[e.cuda_event for e in self.events])
        self.start = torch.cuda.Event()
        self.start.record(cur)
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)

    @property
    def k_base(self) -> int:
        return self.own

    @property
    def v_base(self) -> int:
        C, W = self.shape[0], self.shape[1]
        return self.own + C * W * self.block

    def exchange(self, kt: torch.Tensor, vt: torch.Tensor, side: torch.cuda.Stream) -> None:
        """Pack this rank's (B, Tl, H, D) K/V rows and enqueue the pulls (on ``side`` and the copy streams)."""
        import torch.distributed as dist

        from . import _lib

        C, W, B, Tc, H, D = self.shape
        with torch.cuda.stream(side):
            for e in self.events:  # this rank's pulls of the previous call have landed
                side.wait_event(e)
            dist.all_reduce(self.flag, group=self.group)  # ... and every peer's: safe to overwrite own blocks
            for t, x in ((0, kt), (1, vt)):
                if x.stride(3) != 1 or x.stride(2) != D or x.stride(1) != H * D:
                    x = x.contiguous()
                _lib.check(self.lib.wf_pack_row_blocks(
                    self.own + t * C * W * self.block, x.data_ptr(), B, C * Tc, H * D * self.esz,
                    x.stride(0) * self.esz, C, W * self.block, self.block, self.rank, side.cuda_stream))
            dist.all_reduce(self.flag, group=self.group)  # every rank's own blocks are packed
            self.start.record(side)
        _lib.check(self.lib.wf_peer_pull_blocks(
            self.bases, W, self.rank, C, 2, self.block, self.block, W * self.block, C * W * self.block,
            self.start.cuda_event, self.stream_ptrs, len(self.streams), self.event_ptrs))

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it)."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)  # no rank still pulls
        for p in self.opened:
            self.lib.wf_peer_buffer_close(p)
        self.opened = []
        dist.barrier(group=self.group)  # every rank has unmapped this rank's buffer
        if self.own:
            self.lib.wf_peer_buffer_free(self.own)
            self.own = None


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
                 chunks: int | None = None, transport: str = "peer"):
        if transport not in ("peer", "nccl"):
            raise ValueError(f"transport must be 'peer' or 'nccl', got {transport!r}")
        self.top_k = top_k
        self.scale = scale
        self.tile = tile
        self.group = group
        self.pad_mode = pad_mode
        self.chunks = chunks
        self.transport = transport
        # persistent per-shape gather buffers and side stream: a forward allocates nothing large
        self._kg = None
        self._vg = None
        self._peer = None
        self._side = None

    def _n_chunks(self, Tl: int, world: int) -> int:
        # NCCL transport: one chunk on 2 ranks, where retrieval already hides the gather,
        # 4 chunks from 4 ranks up, where each rank receives (W-1)/W of K/V while its
        # retrieval shrinks as 1/W (cfg4 on 8 GPUs: 3.04 ms in 4 chunks, 3.10 in 2,
        # 3.75 in 8: smaller all-gathers run at lower bandwidth).
        # Peer transport: one chunk on 2 ranks (the pulls hide behind retrieval), 4 from
        # 4 ranks up: the pulls land chunk by chunk, in order, on one copy stream, so
        # the attention of a chunk starts while later chunks arrive.
        if self.chunks is not None:
            want = self.chunks
        elif self.transport == "peer":
            want = 1 if world <= 2 else 4
        else:
            want = 1 if world <= 2 else 4
        c = max(1, min(want, 64 // world, Tl // self.tile))
        while c > 1 and Tl % (c * self.tile):
            c -= 1
        return c

    def close(self) -> None:
        """Release the peer buffers (collective: every rank of the group calls it)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

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
        dev = q_l.device
        main = torch.cuda.current_stream(dev)
        if self._side is None or self._side.device != dev:
            self._side = torch.cuda.Stream(device=dev)
        side = self._side
        shape = (C, world, B, Tc, H, D)
        kt, vt = k_l.transpose(1, 2), v_l.transpose(1, 2)  # (B, Tl, H, D)
        # The key addresses (small) go first: collectives of one process group run in
        # issue order, so issued after the K/V exchange the retrieval would wait for it.
        k_addr = gather_sequence(k_addr_l, self.tile, self.group)  # reordered to global order
        side.wait_stream(main)  # the previous call's attention has finished with the buffers
        if self.transport == "peer":
            if self._peer is None or self._peer.shape != shape or self._peer.dtype != k_l.dtype:
                self.close()
                self._peer = _PeerKV(shape, k_l.dtype, dev, self.group)
            peer = self._peer
            peer.exchange(kt, vt, side)
            idx = sharded_causal_topk(q_addr_l, k_addr, self.top_k, world, rank, self.tile, self.pad_mode)
            out = _chunked_attention(q_l, idx, peer.k_base, peer.v_base, shape, self.scale, self.tile,
                                     self.pad_mode, out_dtype,
                                     wait=lambda c, every: [main.wait_event(e) for e in
                                                            (peer.events if every else peer.events[:c + 1])])
            return out, idx
        if self._kg is None or tuple(self._kg.shape) != shape or self._kg.dtype != k_l.dtype or self._kg.device != dev:
            self._kg = torch.empty(shape, dtype=k_l.dtype, device=dev)
            self._vg = torch.empty(shape, dtype=v_l.dtype, device=dev)
        k_g, v_g = self._kg, self._vg
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
                                   wait=lambda c, every: main.wait_event(landed[-1] if every else landed[c]))
        return out, idx

    __call__ = forward
