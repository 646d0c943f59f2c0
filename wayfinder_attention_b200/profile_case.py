"""Run one hot-path op a few times on synthetic inputs, for profiler captures.

    python -m wayfinder_attention_b200.profile_case --op attention --config cfg2 --iters 3
    python -m wayfinder_attention_b200.profile_case --op topk --config cfg2 --iters 3

Inputs come from ``workloads.make_inputs`` (seeded); a 256 MiB memset before each
call flushes the L2, like the timed steps of ``bench.py``.  Prints nothing but a
final ``ok`` line, so it is safe to run under ncu.
"""

from __future__ import annotations

import argparse

import torch

from .causal_topk import causal_topk
from .fused_sparse import sparse_meat_attention
from .workloads import CONFIGS, make_inputs, to_device


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["topk", "attention", "both"], default="both")
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    w = CONFIGS[a.config]
    x = to_device(make_inputs(w), "cuda:0")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda:0")
    idx = causal_topk(x["q_addr"], x["k_addr"], w.K)
    for _ in range(a.iters):
        flush.zero_()
        if a.op in ("topk", "both"):
            idx = causal_topk(x["q_addr"], x["k_addr"], w.K)
        if a.op in ("attention", "both"):
            sparse_meat_attention(x["q"], x["k"], x["v"], idx, w.D ** -0.5)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
