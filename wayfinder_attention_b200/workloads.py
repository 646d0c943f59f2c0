"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

Configs (B batch, H heads, T sequence, D head_dim, R address dim, K budget):
  cfg1  B=1  H=4  T=2048  D=64  R=32 K=128 fp32   (CPU-runnable reference case)
  cfg2  B=1  H=8  T=16384 D=64  R=32 K=128 bf16   (headline: T=16K, K=128)
  cfg3  4-layer decoder, d_model=256, H=4, D=64, FFN 1024, vocab 128, B=8, T=4096, K=128 bf16
  cfg4  B=1  H=32 T=65536 D=128 R=32 K=128 bf16   (long single sequence, query-row sharded)
  cfg5  B=64 H=16 T=8192  D=64  R=32 K in {64,128,256} bf16, clustered addresses

Values: q, k, v ~ N(0, 1); addresses ~ N(0, 1/32), or for cfg5 a mixture of 64
Gaussian clusters (centres ~ N(0, 1/32), sigma 0.05, cluster uniform per token).
Everything is drawn on the CPU from ``torch.Generator().manual_seed(seed)`` so
the GPU run and any CPU check see identical values.  q/k/v are generated in the
(B, T, H, D) memory layout that ``LearnedAddressSparseAttention`` produces
(``routing_attention/models/attention.py:464-466``) and returned as
(B, H, T, D) views of it.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

SEED = 45


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    T: int
    D: int
    R: int
    K: int
    dtype: torch.dtype
    clustered: bool = False

    @property
    def queries(self) -> int:
        """Token positions per call (the unit of the queries/s metric)."""
        return self.B * self.T

    def score_flops(self) -> float:
        """Causal address-score FLOPs: 2 * B * R * T(T+1)/2 (addresses shared by heads)."""
        return 2.0 * self.B * self.R * self.T * (self.T + 1) / 2

    def gathered_bytes(self) -> float:
        """K and V rows gathered, counted every time: 2 * B * H * T * K * D * sizeof."""
        esz = torch.empty((), dtype=self.dtype).element_size()
        return 2.0 * self.B * self.H * self.T * self.K * self.D * esz

    def compulsory_bytes(self) -> float:
        """Read q/k/v + addresses once, write out + indices once."""
        esz = torch.empty((), dtype=self.dtype).element_size()
        qkvo = 4.0 * self.B * self.H * self.T * self.D * esz
        addr = 2.0 * self.B * self.T * self.R * esz
        idx = 4.0 * self.B * self.T * self.K
        return qkvo + addr + idx


CONFIGS = {
    "cfg1": Workload("cfg1", 1, 4, 2048, 64, 32, 128, torch.float32),
    "cfg2": Workload("cfg2", 1, 8, 16384, 64, 32, 128, torch.bfloat16),
    "cfg3_layer": Workload("cfg3_layer", 8, 4, 4096, 64, 32, 128, torch.bfloat16),
    "cfg4": Workload("cfg4", 1, 32, 65536, 128, 32, 128, torch.bfloat16),
    "cfg5": Workload("cfg5", 64, 16, 8192, 64, 32, 128, torch.bfloat16, clustered=True),
    "cfg5_k64": Workload("cfg5_k64", 64, 16, 8192, 64, 32, 64, torch.bfloat16, clustered=True),
    "cfg5_k256": Workload("cfg5_k256", 64, 16, 8192, 64, 32, 256, torch.bfloat16, clustered=True),
}


def scaled(w: Workload, **kw) -> Workload:
    return replace(w, **kw)


def make_addresses(w: Workload, gen: torch.Generator, B: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    B = w.B if B is None else B
    if w.clustered:
        centres = torch.randn(64, w.R, generator=gen) / math.sqrt(32.0)
        qa = centres[torch.randint(0, 64, (B, w.T), generator=gen)] + 0.05 * torch.randn(B, w.T, w.R, generator=gen)
        ka = centres[torch.randint(0, 64, (B, w.T), generator=gen)] + 0.05 * torch.randn(B, w.T, w.R, generator=gen)
    else:
        qa = torch.randn(B, w.T, w.R, generator=gen) / math.sqrt(32.0)
        ka = torch.randn(B, w.T, w.R, generator=gen) / math.sqrt(32.0)
    return qa.to(w.dtype), ka.to(w.dtype)


def make_inputs(w: Workload, seed: int = SEED, B: int | None = None, batch_offset: int = 0) -> dict:
    """CPU tensors: q_addr, k_addr (B,T,R); q, k, v (B,H,T,D) views of (B,T,H,D) memory.

    ``batch_offset`` seeds a different stream per batch shard so that rank r of a
    batch-sharded run draws its own batch elements.
    """
    B = w.B if B is None else B
    gen = torch.Generator().manual_seed(seed + 1000003 * batch_offset)
    q_addr, k_addr = make_addresses(w, gen, B)
    qkv = [torch.randn(B, w.T, w.H, w.D, generator=gen).to(w.dtype) for _ in range(3)]
    q, k, v = (t.transpose(1, 2) for t in qkv)
    return {"q_addr": q_addr, "k_addr": k_addr, "q": q, "k": k, "v": v}


def to_device(inputs: dict, device) -> dict:
    """Copy preserving the (B,T,H,D) memory layout of q/k/v."""
    out = {}
    for name, t in inputs.items():
        if t.dim() == 4:
            out[name] = t.transpose(1, 2).contiguous().to(device).transpose(1, 2)
        else:
            out[name] = t.contiguous().to(device)
    return out
