"""Sequence-sharded retrieval + attention on 2 GPUs (skipped with fewer): every rank's rows
must equal the same rows of the single-GPU fused call."""

import os
import subprocess
import sys
import textwrap

import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu

SCRIPT = textwrap.dedent(
    """
    import os, sys, torch, torch.distributed as dist
    sys.path.insert(0, %r)
    from wayfinder_attention_b200 import fused_sparse_attention
    from wayfinder_attention_b200.sharding import SequenceShardedAttention, local_rows
    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    B, T, H, D, R, K, tile = 2, 4096, 4, 64, 32, 128, 256
    g = torch.Generator(device=dev).manual_seed(45)
    qa = (torch.randn(B, T, R, generator=g, device=dev) / 32 ** 0.5).bfloat16()
    ka = (torch.randn(B, T, R, generator=g, device=dev) / 32 ** 0.5).bfloat16()
    qkv = [torch.randn(B, T, H, D, generator=g, device=dev).bfloat16() for _ in range(3)]
    full_out, full_idx = fused_sparse_attention(qa, ka, *(t.transpose(1, 2) for t in qkv), K, D ** -0.5)
    rows = torch.from_numpy(local_rows(T, world, rank, tile)).to(dev)
    ok = True
    for transport in ("nccl", "peer"):
        for chunks in (8, 1):  # 8 K/V chunks of 256 local rows, or one
            op = SequenceShardedAttention(K, D ** -0.5, tile=tile, chunks=chunks, transport=transport)
            local = [t[:, rows].contiguous().transpose(1, 2) for t in qkv]
            # a first call on other K/V, then the real one reusing the exchange buffers:
            # a pull or pack racing across the two calls would show in the second result
            op(qa[:, rows].contiguous(), ka[:, rows].contiguous(), local[0], local[1] * 3, local[2] * -2)
            out, idx = op(qa[:, rows].contiguous(), ka[:, rows].contiguous(), *local)
            torch.cuda.synchronize()
            good = torch.equal(idx, full_idx[:, rows]) and torch.equal(out, full_out[:, :, rows])
            print(f"rank {rank} {transport} chunks={chunks} ok={good}", flush=True)
            ok = ok and good
            op.close()
    dist.barrier(); dist.destroy_process_group()
    sys.exit(0 if ok else 1)
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_sharded_matches_single_gpu(tmp_path):
    script = tmp_path / "seq_shard.py"
    script.write_text(SCRIPT % str(REPO))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
         "--master-addr=127.0.0.1", "--master-port=29531", str(script)],
        capture_output=True, text=True, timeout=300, env=env,
    )
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
