"""Generate the golden fixtures under tests/golden/ by running the REFERENCE itself.

Run in a container where the reference checkout is importable:

    WF_REFERENCE_PATH=/path/to/wayfinder-attention python tests/golden/make_golden.py

For every case it draws seeded inputs, calls the reference's own path on CPU in
fp32 -- ``routing_attention.kernels.fused_sparse.fused_sparse_attention(q_addr,
k_addr, q, k, v, K, D**-0.5, retrieval_method="fused_causal")`` (which runs
``_causal_topk_row_blocked`` + ``sparse_meat_attention_reference``) -- and
stores its indices and outputs.  bf16 cases hold bf16-valued inputs upcast to
fp32 (the reference upcasts addresses itself, causal_topk.py:150-151).

Small cases store their inputs; larger ones store a SHA-256 of the inputs that
``wayfinder_attention_b200.workloads.make_inputs`` regenerates from the seed,
plus the full index tensor and a subset of output rows.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from wayfinder_attention_b200.workloads import CONFIGS, Workload, make_inputs  # noqa: E402

CASES = [
    # name, workload, store_inputs
    ("small_f32", Workload("small_f32", 2, 2, 300, 16, 32, 16, torch.float32), True),
    ("short_seq", Workload("short_seq", 1, 2, 100, 16, 32, 128, torch.float32), True),
    ("clustered_ties", Workload("clustered_ties", 1, 2, 512, 32, 32, 64, torch.float32, clustered=True), True),
    ("bf16_t1024", Workload("bf16_t1024", 1, 8, 1024, 64, 32, 128, torch.bfloat16), False),
    ("cfg1", CONFIGS["cfg1"], False),
]


def input_digest(inp: dict) -> str:
    h = hashlib.sha256()
    for name in ("q_addr", "k_addr", "q", "k", "v"):
        h.update(inp[name].float().contiguous().numpy().tobytes())
    return h.hexdigest()


def out_rows(T: int, K: int) -> np.ndarray:
    """Output rows kept for large cases: every pad row, then every 16th row."""
    return np.unique(np.concatenate([np.arange(min(K, T)), np.arange(0, T, 16), [T - 1]]))


def main() -> None:
    ref = os.environ.get("WF_REFERENCE_PATH", "/root/reference")
    sys.path.insert(0, ref)
    from routing_attention.kernels.fused_sparse import fused_sparse_attention  # reference code

    torch.set_num_threads(os.cpu_count() or 1)
    for name, w, store_inputs in CASES:
        inp = make_inputs(w, seed=45)
        f32 = {k: v.float() for k, v in inp.items()}
        scale = w.D ** -0.5
        out, idx = fused_sparse_attention(
            f32["q_addr"], f32["k_addr"], f32["q"], f32["k"], f32["v"], w.K, scale, retrieval_method="fused_causal"
        )
        rec = {
            "B": w.B, "H": w.H, "T": w.T, "D": w.D, "R": w.R, "K": w.K,
            "dtype": str(w.dtype).replace("torch.", ""), "clustered": int(w.clustered), "seed": 45,
            "scale": scale, "digest": input_digest(inp),
            "idx": idx.numpy().astype(np.int32),
        }
        if store_inputs:
            for k_, v_ in f32.items():
                rec[k_] = v_.contiguous().numpy()
            rec["out"] = out.numpy()
            rec["out_rows"] = np.arange(w.T)
        else:
            rows = out_rows(w.T, w.K)
            rec["out"] = out[:, :, rows].numpy()
            rec["out_rows"] = rows
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(name, "idx", tuple(idx.shape), "out", tuple(rec["out"].shape))


if __name__ == "__main__":
    main()
