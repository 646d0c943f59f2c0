"""Routing-vector producers for ``RoutingSparseAttention``.

Drop-ins for ``routing_attention/models/router.py``: ``RouterMLP`` (:12-115),
``PerLayerRouter`` (:118-156) and ``MultiScaleRouter`` (:159-207), with the same
constructor arguments and submodule names (``net``, ``key_net``, ``dot_scale``,
``dot_bias``, ``routers``, ``local_router``, ``global_router``) so reference
``state_dict``s load unchanged.  The MLPs are small dense layers and stay in
PyTorch; their output (B, T, R) routing vectors are the search vectors of the
fused retrieval + sparse-attention kernels.
"""

from __future__ import annotations

from typing import Literal

import torch
import torch.nn as nn
import torch.nn.functional as F

from .causal_topk import causal_topk


class RouterMLP(nn.Module):
    """Maps hidden states to routing vectors (``router.py:12-115``).

    symmetric: one vector r_i per token, similarity r_i . r_j;
    asymmetric: separate query and key vectors, similarity q_i . k_j.
    """

    def __init__(
        self,
        input_dim: int,
        routing_dim: int = 32,
        hidden_dim: int | None = None,
        normalize: bool = True,
        dropout: float = 0.0,
        use_affine_dot: bool = False,
        similarity: Literal["symmetric", "asymmetric"] = "symmetric",
        n_heads: int = 1,
        per_head_routing: bool = False,
    ):
        super().__init__()
        hidden_dim = hidden_dim or max(routing_dim * 2, input_dim // 4)
        self.normalize = normalize
        self.use_affine_dot = use_affine_dot
        self.similarity = similarity
        self.n_heads = n_heads
        self.per_head_routing = per_head_routing
        self.routing_dim = routing_dim
        out_dim = routing_dim * n_heads if per_head_routing else routing_dim

        def mlp() -> nn.Sequential:
            return nn.Sequential(nn.Linear(input_dim, hidden_dim), nn.GELU(), nn.Dropout(dropout),
                                 nn.Linear(hidden_dim, out_dim))

        self.net = mlp()
        if similarity == "asymmetric":
            self.key_net = mlp()
        if use_affine_dot:
            self.dot_scale = nn.Parameter(torch.tensor(1.0))
            self.dot_bias = nn.Parameter(torch.tensor(0.0))

    def forward(self, x: torch.Tensor, as_query: bool = True) -> torch.Tensor:
        """(B, T, R) routing vectors, or (B, T, H, R) with per-head routing."""
        r = self.key_net(x) if (self.similarity == "asymmetric" and not as_query) else self.net(x)
        if self.per_head_routing:
            B, T, _ = r.shape
            r = r.view(B, T, self.n_heads, self.routing_dim)
        return F.normalize(r, dim=-1) if self.normalize else r

    def forward_query_key(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        q = self.forward(x, as_query=True)
        k = self.forward(x, as_query=False) if self.similarity == "asymmetric" else q
        return q, k


class PerLayerRouter(nn.Module):
    """One ``RouterMLP`` per transformer layer (``router.py:118-156``)."""

    def __init__(self, n_layers: int, input_dim: int, routing_dim: int = 32, hidden_dim: int | None = None,
                 normalize: bool = True, use_affine_dot: bool = False, similarity: str = "symmetric",
                 n_heads: int = 1, per_head_routing: bool = False):
        super().__init__()
        self.n_layers = n_layers
        self.routers = nn.ModuleList([
            RouterMLP(input_dim, routing_dim, hidden_dim, normalize, use_affine_dot=use_affine_dot,
                      similarity=similarity, n_heads=n_heads, per_head_routing=per_head_routing)
            for _ in range(n_layers)
        ])

    def forward(self, x: torch.Tensor, layer_idx: int, as_query: bool = True) -> torch.Tensor:
        return self.routers[layer_idx](x, as_query=as_query)

    def forward_query_key(self, x: torch.Tensor, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.routers[layer_idx].forward_query_key(x)


class MultiScaleRouter(nn.Module):
    """Local + global routers (``router.py:159-207``).

    ``forward`` concatenates both normalised routing vectors (the search vectors the
    fused path uses, R = 2 * routing_dim).  ``retrieve_indices`` runs the causal
    top-K kernel once per router (K/2 and K - K/2) and merges the two candidate
    sets per row as the reference does: ascending unique indices, short rows
    filled with their smallest index.
    """

    def __init__(self, input_dim: int, routing_dim: int = 32, hidden_dim: int | None = None,
                 local_window: int = 16, similarity: str = "symmetric", n_heads: int = 1,
                 per_head_routing: bool = False):
        super().__init__()
        hidden_dim = hidden_dim or max(routing_dim * 2, input_dim // 4)
        self.local_window = local_window
        kw = dict(similarity=similarity, n_heads=n_heads, per_head_routing=per_head_routing)
        self.local_router = RouterMLP(input_dim, routing_dim, hidden_dim, normalize=True, **kw)
        self.global_router = RouterMLP(input_dim, routing_dim, hidden_dim, normalize=True, **kw)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return torch.cat([self.local_router(x), self.global_router(x)], dim=-1)

    def retrieve_indices(self, x: torch.Tensor, k: int, layer_idx: int = 0) -> torch.Tensor:
        """(B, T, k) int64 merged candidates (``router.py:185-204``), vectorised."""
        del layer_idx
        k_half = max(1, k // 2)
        parts = []
        for router, kk in ((self.local_router, k_half), (self.global_router, k - k_half)):
            if kk <= 0:
                continue
            q, kv = router.forward_query_key(x)
            parts.append(causal_topk(q, kv, kk).long())
        cand = torch.cat(parts, dim=-1)
        srt, _ = torch.sort(cand, dim=-1)
        dup = torch.zeros_like(srt, dtype=torch.bool)
        dup[..., 1:] = srt[..., 1:] == srt[..., :-1]
        # unique values first (stable order of the sorted row), duplicates after
        order = torch.argsort(dup.to(torch.int8), dim=-1, stable=True)
        uniq = torch.gather(srt, -1, order)
        n = (~dup).sum(-1, keepdim=True)
        pos = torch.arange(cand.shape[-1], device=cand.device)
        merged = torch.where(pos < n, uniq, srt[..., :1])
        if merged.shape[-1] < k:
            merged = torch.cat([merged, srt[..., :1].expand(*merged.shape[:-1], k - merged.shape[-1])], dim=-1)
        return merged[..., :k]
