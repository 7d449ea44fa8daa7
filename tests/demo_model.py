"""Torch modules with the structure of the reference demo model (demo.py:41-140).

The reference demo's layers are user code wrapped by FoldedModel; these are
the same layers (post-norm MHA + GELU FFN) written for the tests, loaded with
the seeded weights of ``actfold_b200.workloads.demo_weights``.
"""

from __future__ import annotations

import torch
import torch.nn as nn


class SyntheticTransformerLayer(nn.Module):
    def __init__(self, hidden_dim: int, num_heads: int) -> None:
        super().__init__()
        self.attn = nn.MultiheadAttention(embed_dim=hidden_dim, num_heads=num_heads, batch_first=True)
        self.norm1 = nn.LayerNorm(hidden_dim)
        self.ffn = nn.Sequential(nn.Linear(hidden_dim, hidden_dim * 4), nn.GELU(), nn.Linear(hidden_dim * 4, hidden_dim))
        self.norm2 = nn.LayerNorm(hidden_dim)

    def forward(self, hidden_states: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        x, _ = self.attn(hidden_states, hidden_states, hidden_states, attn_mask=attention_mask)
        x = self.norm1(x + hidden_states)
        return self.norm2(self.ffn(x) + x)


class SyntheticTransformer(nn.Module):
    def __init__(self, vocab_size: int = 1000, hidden_dim: int = 128, num_layers: int = 4, num_heads: int = 8) -> None:
        super().__init__()
        self.embedding = nn.Embedding(vocab_size, hidden_dim)
        self.layers = nn.ModuleList(SyntheticTransformerLayer(hidden_dim, num_heads) for _ in range(num_layers))
        self.lm_head = nn.Linear(hidden_dim, vocab_size, bias=False)

    def forward(self, tokens: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        x = self.embedding(tokens)
        for layer in self.layers:
            x = layer(x, attention_mask=attention_mask)
        return self.lm_head(x)


def load_demo_weights(model: SyntheticTransformer, w: dict) -> SyntheticTransformer:
    t = torch.from_numpy
    with torch.no_grad():
        model.embedding.weight.copy_(t(w["embedding"]))
        model.lm_head.weight.copy_(t(w["lm_head"]))
        for lw, layer in zip(w["layers"], model.layers):
            layer.attn.in_proj_weight.copy_(t(lw["in_proj_weight"]))
            layer.attn.in_proj_bias.copy_(t(lw["in_proj_bias"]))
            layer.attn.out_proj.weight.copy_(t(lw["out_proj_weight"]))
            layer.attn.out_proj.bias.copy_(t(lw["out_proj_bias"]))
            layer.norm1.weight.copy_(t(lw["norm1_weight"]))
            layer.norm1.bias.copy_(t(lw["norm1_bias"]))
            layer.ffn[0].weight.copy_(t(lw["ffn0_weight"]))
            layer.ffn[0].bias.copy_(t(lw["ffn0_bias"]))
            layer.ffn[2].weight.copy_(t(lw["ffn2_weight"]))
            layer.ffn[2].bias.copy_(t(lw["ffn2_bias"]))
            layer.norm2.weight.copy_(t(lw["norm2_weight"]))
            layer.norm2.bias.copy_(t(lw["norm2_bias"]))
    return model
