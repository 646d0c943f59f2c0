"""Generate the decoder and non-fused-module golden fixtures from the REFERENCE on CPU.

    WF_REFERENCE_PATH=/path/to/wayfinder-attention python tests/golden/make_golden_models.py

Cases:
  * ``decoder_learned_address.npz``: the reference ``TransformerLM``
    (``routing_attention/models/transformer.py:76-401``) with
    ``attention_type="learned_address"`` on the fused path, 2 layers, d_model 64,
    4 heads, FFN 128, vocab 128, K=16; token ids (2, 160), every ``state_dict``
    entry (``sd/``) and the logits, eval mode, fp32.
  * ``modules_learned_address_nonfused.npz``: ``LearnedAddressSparseAttention``
    on the non-fused path (``use_fused_sparse`` off, method ``fused_causal``):
    addresses cast to fp16 before the retrieval (``retrieval/index.py:188-207``),
    then gather + softmax + weighted sum (``models/attention.py:35-56``).

Slot convention.  The reference's CPU path fills the pad slots of rows t < K-1
according to the unsorted slot order of ``torch.topk(sorted=False)``
(``kernels/causal_topk.py:37-57``, ``:167``), which is implementation-defined; its
Triton path sorts the slots first (``:432-434``) and the pads then occupy slots
t+1..K-1.  In a multi-layer model the pad rows feed later layers, so this script
runs the reference with the Triton path's convention: ``_finalize_causal_topk`` is
wrapped to sort each row by descending score before the reference's own pad fix.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _sorted_slot_convention():
    import importlib

    # (the package re-exports a function of the same name, so no attribute import)
    ct = importlib.import_module("routing_attention.kernels.causal_topk")
    original = ct._finalize_causal_topk

    def finalize_sorted(out_val, out_idx, k_eff):
        vals, order = torch.sort(out_val[..., :k_eff], dim=-1, descending=True, stable=True)
        return original(vals, out_idx[..., :k_eff].gather(-1, order), k_eff)

    ct._finalize_causal_topk = finalize_sorted


def _save(name, rec, model):
    for k, v in model.state_dict().items():
        rec["sd/" + k] = v.numpy()
    np.savez_compressed(HERE / f"{name}.npz", **rec)
    print(name, len([k for k in rec if k.startswith("sd/")]), "state entries")


def main() -> None:
    sys.path.insert(0, os.environ.get("WF_REFERENCE_PATH", "/root/reference"))
    _sorted_slot_convention()
    from routing_attention.models.attention import LearnedAddressSparseAttention
    from routing_attention.models.transformer import TransformerLM

    torch.manual_seed(300)
    lm = TransformerLM(128, d_model=64, n_layers=2, n_heads=4, d_ff=128, max_seq_len=192, dropout=0.1,
                       attention_type="learned_address", routing_top_k=16,
                       retrieval_config={"use_fused_sparse": True, "method": "fused_causal"}).eval()
    ids = torch.randint(0, 128, (2, 160), generator=torch.Generator().manual_seed(301))
    with torch.no_grad():
        logits = lm(ids)["logits"]
    _save("decoder_learned_address", {"ids": ids.numpy(), "logits": logits.numpy(),
                                      "meta/top_k": np.array(16)}, lm)

    torch.manual_seed(302)
    m = LearnedAddressSparseAttention(64, 4, top_k=16, address_dim=32,
                                      retrieval_config={"method": "fused_causal"}).eval()
    x = torch.randn(2, 160, 64, generator=torch.Generator().manual_seed(303))
    with torch.no_grad():
        out = m(x)
    _save("modules_learned_address_nonfused", {
        "x": x.numpy(), "out": out.numpy(), "meta/d_model": np.array(64), "meta/n_heads": np.array(4),
        "meta/top_k": np.array(16), "meta/nonfused": np.array(1)}, m)


if __name__ == "__main__":
    main()
