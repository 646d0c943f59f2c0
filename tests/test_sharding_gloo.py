"""Multi-process host logic of the sequence sharding, on CPU with the gloo backend (world size 2)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wayfinder_attention_b200.sharding import gather_sequence, local_rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, tile, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        full = torch.randn(2, T, 3, 4, generator=g)
        rows = torch.from_numpy(local_rows(T, world, rank, tile))
        got = gather_sequence(full[:, rows], tile)
        ok = torch.equal(got, full)
        addr = torch.randn(2, T, 32, generator=g)
        ok = ok and torch.equal(gather_sequence(addr[:, rows], tile), addr)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T,tile", [(2, 1024, 64), (2, 2048, 256)])
def test_gather_sequence_rebuilds_global_order(world, T, tile):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, tile, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {r: True for r in range(world)}


def test_gather_sequence_rejects_partial_blocks():
    # the check happens before any collective, so no process group is needed
    with pytest.raises(ValueError, match="whole number"):
        gather_sequence(torch.zeros(1, 100, 4), 64)


def _dropout_worker(rank, world, port, q):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))  # this rank leaves between steps, before the next collective
        q.close()
        q.join_thread()
        os._exit(0)
    try:
        gather_sequence(torch.zeros(1, 128, 4), 64)
        q.put((rank, "no error"))
    except Exception as e:  # the surviving rank must see an error, not hang
        q.put((rank, type(e).__name__))
    q.close()
    q.join_thread()
    os._exit(0)


def test_missing_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0] != "no error"
