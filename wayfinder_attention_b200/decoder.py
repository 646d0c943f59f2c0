"""Decoder-only LM harness around the Wayfinder attention op (prefill forward).

A compact restatement of the reference's ``TransformerLM`` for the one model
family on the hot path (``routing_attention/models/transformer.py:26-72``
block, ``:76-312`` model): token + learned position embeddings, pre-LN blocks
(``x + attn(ln1(x))``, ``x + ff(ln2(x))`` with a GELU FFN), final LayerNorm and
an LM head tied to the token embedding.  Parameter names match the reference
(``token_emb``, ``pos_emb``, ``blocks.N.attn.*``, ``blocks.N.ln1`` …), so its
``state_dict`` loads.  Only ``attention_type`` "learned_address" (this build's
kernels) and "dense_flash" (PyTorch SDPA, the dense baseline of
``models/attention.py:130-173``) are provided.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import KeyVectorSparseAttention, LearnedAddressSparseAttention


class DenseSDPAAttention(nn.Module):
    """Dense causal attention through ``F.scaled_dot_product_attention`` (``attention.py:130-173``)."""

    def __init__(self, d_model: int, n_heads: int, dropout: float = 0.1):
        super().__init__()
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.dropout_p = dropout

    def forward(self, x: torch.Tensor, attn_mask: Optional[torch.Tensor] = None, **kwargs) -> torch.Tensor:
        B, T, D = x.shape
        q = self.q_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        out = F.scaled_dot_product_attention(
            q, k, v, is_causal=True, scale=self.scale, dropout_p=self.dropout_p if self.training else 0.0
        )
        return self.out_proj(out.transpose(1, 2).contiguous().view(B, T, D))


class TransformerBlock(nn.Module):
    def __init__(self, d_model: int, n_heads: int, d_ff: int, dropout: float, attention_module: nn.Module,
                 layer_idx: int = 0):
        super().__init__()
        self.attn = attention_module
        self.layer_idx = layer_idx
        self.ln1 = nn.LayerNorm(d_model)
        self.ln2 = nn.LayerNorm(d_model)
        self.ff = nn.Sequential(
            nn.Linear(d_model, d_ff), nn.GELU(), nn.Dropout(dropout), nn.Linear(d_ff, d_model), nn.Dropout(dropout)
        )

    def forward(self, x: torch.Tensor, attn_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        x = x + self.attn(self.ln1(x), attn_mask=attn_mask)
        return x + self.ff(self.ln2(x))


class TransformerLM(nn.Module):
    def __init__(
        self,
        vocab_size: int,
        d_model: int = 256,
        n_layers: int = 6,
        n_heads: int = 4,
        d_ff: int = 1024,
        max_seq_len: int = 512,
        dropout: float = 0.1,
        attention_type: str = "learned_address",
        routing_top_k: int = 32,
        address_dim: int = 32,
        retrieval_config: Optional[dict] = None,
        pad_token_id: int = 0,
    ):
        super().__init__()
        if attention_type not in ("learned_address", "key_vector", "dense_flash", "dense"):
            raise ValueError(f"attention_type {attention_type!r} is outside this build's scope")
        self.d_model = d_model
        self.max_seq_len = max_seq_len
        self.pad_token_id = pad_token_id
        self.token_emb = nn.Embedding(vocab_size, d_model)
        self.pos_emb = nn.Embedding(max_seq_len, d_model)
        self.dropout = nn.Dropout(dropout)
        self.blocks = nn.ModuleList()
        for i in range(n_layers):
            if attention_type == "learned_address":
                attn = LearnedAddressSparseAttention(
                    d_model, n_heads, routing_top_k, address_dim=address_dim, dropout=dropout,
                    retrieval_config=retrieval_config,
                )
            elif attention_type == "key_vector":
                attn = KeyVectorSparseAttention(d_model, n_heads, routing_top_k, dropout=dropout,
                                                retrieval_config=retrieval_config)
            else:
                attn = DenseSDPAAttention(d_model, n_heads, dropout)
            self.blocks.append(TransformerBlock(d_model, n_heads, d_ff, dropout, attn, layer_idx=i))
        self.ln_f = nn.LayerNorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        self.lm_head.weight = self.token_emb.weight

    def forward(self, input_ids: torch.Tensor, attn_mask: Optional[torch.Tensor] = None) -> dict:
        B, T = input_ids.shape
        if attn_mask is None:
            attn_mask = input_ids != self.pad_token_id
        pos = torch.arange(T, device=input_ids.device).unsqueeze(0)
        x = self.dropout(self.token_emb(input_ids) + self.pos_emb(pos))
        for block in self.blocks:
            x = block(x, attn_mask=attn_mask)
        return {"logits": self.lm_head(self.ln_f(x))}
