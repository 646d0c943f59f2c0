"""Generate module-level golden fixtures by running the REFERENCE modules on CPU.

    WF_REFERENCE_PATH=/path/to/wayfinder-attention python tests/golden/make_golden_modules.py

Each case builds a reference attention module (fused path,
``retrieval_config={"use_fused_sparse": True, "method": "fused_causal"}``) with
seeded random weights, runs it in eval mode on a seeded input in fp32, and stores
the input, every ``state_dict`` entry (prefixed ``sd/``) and the output in
``modules_<case>.npz``.  The drop-in modules load the same ``state_dict`` and must
reproduce the output (``tests/test_gpu_modules_golden.py``).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

FUSED = {"use_fused_sparse": True, "method": "fused_causal"}


def cases(ref):
    from routing_attention.models.attention import (
        KeyVectorSparseAttention,
        LearnedAddressSparseAttention,
        RoutingSparseAttention,
    )
    from routing_attention.models.router import MultiScaleRouter, PerLayerRouter, RouterMLP

    yield "learned_address", dict(d_model=64, n_heads=4, top_k=16), lambda: LearnedAddressSparseAttention(
        64, 4, top_k=16, address_dim=32, retrieval_config=dict(FUSED))
    yield "key_vector", dict(d_model=64, n_heads=2, top_k=24), lambda: KeyVectorSparseAttention(
        64, 2, top_k=24, retrieval_config=dict(FUSED))
    yield "routing_asym", dict(d_model=64, n_heads=4, top_k=16, router="mlp_asym"), lambda: RoutingSparseAttention(
        64, 4, RouterMLP(64, 32, similarity="asymmetric"), top_k=16, retrieval_config=dict(FUSED))
    yield "routing_per_layer", dict(d_model=64, n_heads=4, top_k=16, router="per_layer", layer_idx=1), \
        lambda: RoutingSparseAttention(64, 4, PerLayerRouter(2, 64, 32, similarity="symmetric"), top_k=16,
                                       layer_idx=1, retrieval_config=dict(FUSED))
    yield "routing_multi_scale", dict(d_model=64, n_heads=4, top_k=16, router="multi_scale"), \
        lambda: RoutingSparseAttention(64, 4, MultiScaleRouter(64, 16), top_k=16, retrieval_config=dict(FUSED))


def main() -> None:
    ref = os.environ.get("WF_REFERENCE_PATH", "/root/reference")
    sys.path.insert(0, ref)
    for i, (name, meta, build) in enumerate(cases(ref)):
        torch.manual_seed(100 + i)
        m = build().eval()
        g = torch.Generator().manual_seed(200 + i)
        x = torch.randn(2, 160, meta["d_model"], generator=g)
        with torch.no_grad():
            out = m(x)
        rec = {"x": x.numpy(), "out": out.numpy()}
        for k, v in m.state_dict().items():
            rec["sd/" + k] = v.numpy()
        for k, v in meta.items():
            rec["meta/" + k] = np.array(v)
        np.savez_compressed(HERE / f"modules_{name}.npz", **rec)
        print(name, tuple(out.shape), len([k for k in rec if k.startswith("sd/")]), "state entries")


if __name__ == "__main__":
    main()
