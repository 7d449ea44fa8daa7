"""demo.py's synthetic Transformer restated in numpy, float32 (TEST INFRASTRUCTURE).

Follows demo.py:41-97: SyntheticTransformerLayer is POST-norm,
``x1 = LN1(MHA(x) + x)``, ``out = LN2(W2 gelu(W1 x1 + b1) + b2 + x1)``,
with torch.nn.MultiheadAttention (batch_first, packed in_proj) and exact
(erf) GELU; SyntheticTransformer is embedding -> layers -> bias-free lm_head.
"""

from __future__ import annotations

import math

import numpy as np

from oracle.folding import folded_layer


def _erf(x: np.ndarray) -> np.ndarray:
    v = np.vectorize(math.erf, otypes=[np.float64])
    return v(x.astype(np.float64)).astype(np.float32)


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    mu = x.mean(-1, keepdims=True, dtype=np.float32)
    var = ((x - mu) ** 2).mean(-1, keepdims=True, dtype=np.float32)
    return ((x - mu) / np.sqrt(var + np.float32(eps)) * w + b).astype(np.float32)


def mha(x: np.ndarray, lw: dict, n_heads: int) -> np.ndarray:
    T, H = x.shape
    d = H // n_heads
    qkv = x @ lw["in_proj_weight"].T + lw["in_proj_bias"]
    q, k, v = qkv[:, :H], qkv[:, H : 2 * H], qkv[:, 2 * H :]
    out = np.empty((T, H), np.float32)
    for h in range(n_heads):
        sl = slice(h * d, (h + 1) * d)
        s = (q[:, sl] @ k[:, sl].T) / np.float32(math.sqrt(d))
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(-1, keepdims=True)
        out[:, sl] = p @ v[:, sl]
    return (out @ lw["out_proj_weight"].T + lw["out_proj_bias"]).astype(np.float32)


def layer(x: np.ndarray, lw: dict, n_heads: int) -> np.ndarray:
    x1 = layer_norm(mha(x, lw, n_heads) + x, lw["norm1_weight"], lw["norm1_bias"])
    f = x1 @ lw["ffn0_weight"].T + lw["ffn0_bias"]
    f = (0.5 * f * (1.0 + _erf(f / np.float32(math.sqrt(2.0))))).astype(np.float32)
    f = f @ lw["ffn2_weight"].T + lw["ffn2_bias"]
    return layer_norm(f + x1, lw["norm2_weight"], lw["norm2_bias"])


def forward(tokens: np.ndarray, weights: dict, n_heads: int) -> dict:
    x = weights["embedding"][tokens]
    states = [x]
    for lw in weights["layers"]:
        x = layer(x, lw, n_heads)
        states.append(x)
    return {"layer_in": np.stack(states), "logits": (x @ weights["lm_head"].T).astype(np.float32)}


def folded_children(children: np.ndarray, parent: dict, weights: dict, n_heads: int, tau: float) -> dict:
    """Folded verification of each child [C, T] against the parent (fp32 gate)."""
    C, T = children.shape
    n_layers = len(weights["layers"])
    masks = np.zeros((n_layers, C, T), bool)
    logits = []
    for c in range(C):
        h = weights["embedding"][children[c]][None]
        for li, lw in enumerate(weights["layers"]):
            fn = lambda x, lw=lw: layer(x, lw, n_heads)  # noqa: E731
            h, m = folded_layer(fn, h, parent["layer_in"][li][None], parent["layer_in"][li + 1][None], tau, "f32")
            masks[li, c] = m[0]
        logits.append(h[0] @ weights["lm_head"].T)
    return {"masks": masks, "logits": np.stack(logits).astype(np.float32)}
