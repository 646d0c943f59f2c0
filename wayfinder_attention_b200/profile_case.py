"""Run one hot-path op a few times on synthetic inputs, for profiler captures.

    python -m wayfinder_attention_b200.profile_case --op attention --config cfg2 --iters 3
    python -m wayfinder_attention_b200.profile_case --op topk --config cfg2 --iters 3
    python -m wayfinder_attention_b200.profile_case --op backward --config cfg2 --iters 3
    python -m wayfinder_attention_b200.profile_case --op projection --iters 3

``projection`` runs the fused address projection of the decoder's shape
(32768 x 256 bf16 hidden states, d_A = 32, both addresses).

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
    ap.add_argument("--op", choices=["topk", "attention", "both", "backward", "projection"], default="both")
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda:0")
    if a.op == "projection":
        from .address_projection import address_projection

        g = torch.Generator().manual_seed(45)
        hid = torch.randn(32768, 256, generator=g).to(torch.bfloat16).to("cuda:0")
        wgt = (torch.randn(64, 256, generator=g) / 16).to(torch.bfloat16).to("cuda:0")
        bias = torch.zeros(64, dtype=torch.bfloat16, device="cuda:0")
        for _ in range(a.iters):
            flush.zero_()
            address_projection(hid, wgt, bias, 32)
        torch.cuda.synchronize()
        print("ok")
        return
    w = CONFIGS[a.config]
    x = to_device(make_inputs(w), "cuda:0")
    idx = causal_topk(x["q_addr"], x["k_addr"], w.K)
    for _ in range(a.iters):
        flush.zero_()
        if a.op in ("topk", "both"):
            idx = causal_topk(x["q_addr"], x["k_addr"], w.K)
        if a.op in ("attention", "both"):
            sparse_meat_attention(x["q"], x["k"], x["v"], idx, w.D ** -0.5)
        if a.op == "backward":
            from .fused_sparse import _launch_attention_backward

            _launch_attention_backward(x["q"], x["k"], x["v"], idx, x["q"], w.D ** -0.5, False)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
