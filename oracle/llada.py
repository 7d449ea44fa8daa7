"""LLaDA-architecture Transformer restated in numpy (TEST INFRASTRUCTURE).

No LLaDA/Dream layer code ships with the reference (its models are loaded via
Hugging Face ``trust_remote_code``), so this module restates the
architecture the workloads name: pre-norm blocks with RMSNorm, RoPE
(rotate-half convention), non-causal multi-head / grouped-query attention and
a SwiGLU FFN, all in bf16 storage with float32 arithmetic. Each named tensor
below is rounded to bf16 once, at the point the CUDA kernels round it:

    a    = rnd(rnd(x * rsqrt(mean(x^2) + eps)) * w_attn_norm)
    q,k,v= rnd(a @ W^T)                      (f32 accumulation)
    q,k  = rnd(rope(q)), rnd(rope(k))         (f32 math on the bf16 values)
    o    = rnd(softmax(q k^T / sqrt(d)) v)    (f32 scores and weights)
    h    = rnd(x + rnd(o @ Wo^T))
    b    = rnd(rnd(h * rsqrt(mean(h^2) + eps)) * w_ffn_norm)
    f    = rnd(silu(rnd(b @ Wg^T)) * rnd(b @ Wu^T))
    out  = rnd(h + rnd(f @ Wd^T))
    logits = rnd(rnd(norm(x_L)) @ W_lm^T)

The folding semantics applied on top (parent pass, then per-child gate →
parent output for stable rows / recomputed output for divergent rows) follow
actfold/core/folded_transformer.py:60-203 and live in ``oracle.folding``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.numerics import round_bf16 as rnd


@dataclass(frozen=True)
class LLaDADims:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rms_eps: float = 1e-5
    rope_theta: float = 500000.0


def rope_tables(T: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin tables [T, head_dim/2] in float32.

    angle(t, i) = t * theta ** (-2 i / d), evaluated in float64 and rounded
    once to float32 after cos/sin.
    """
    inv = 1.0 / (float(theta) ** (np.arange(0, head_dim, 2, dtype=np.float64) / float(head_dim)))
    ang = np.arange(T, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    xn = rnd(x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))))
    return rnd(xn * w)


def apply_rope(x: np.ndarray, pos: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x: [T, n, d] bf16 values; rotate-half RoPE at positions ``pos``."""
    d = x.shape[-1]
    h = d // 2
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    x1, x2 = x[..., :h], x[..., h:]
    out = np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)
    return rnd(out)


def silu(x: np.ndarray) -> np.ndarray:
    return x / (np.float32(1.0) + np.exp(-x))


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, dims: LLaDADims) -> np.ndarray:
    """Non-causal attention. q: [Tq, nh, d], k/v: [Tk, nkv, d] -> [Tq, nh*d] (bf16 values)."""
    nh, nkv, d = dims.n_heads, dims.n_kv_heads, dims.head_dim
    grp = nh // nkv
    scale = np.float32(1.0 / np.sqrt(d))
    out = np.empty((q.shape[0], nh, d), np.float32)
    for h in range(nh):
        g = h // grp
        s = (q[:, h, :] @ k[:, g, :].T) * scale
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(axis=-1, keepdims=True)
        out[:, h, :] = rnd(p @ v[:, g, :])
    return out.reshape(q.shape[0], nh * d)


def block(x: np.ndarray, lw: dict, dims: LLaDADims, cos: np.ndarray, sin: np.ndarray, return_kv: bool = False):
    """One LLaDA block on a full sequence x: [T, H] (bf16 values)."""
    T = x.shape[0]
    nh, nkv, d = dims.n_heads, dims.n_kv_heads, dims.head_dim
    pos = np.arange(T)
    a = rmsnorm(x, lw["attn_norm"], dims.rms_eps)
    q = rnd(a @ lw["wq"].T).reshape(T, nh, d)
    k = rnd(a @ lw["wk"].T).reshape(T, nkv, d)
    v = rnd(a @ lw["wv"].T).reshape(T, nkv, d)
    q = apply_rope(q, pos, cos, sin)
    k = apply_rope(k, pos, cos, sin)
    o = attention(q, k, v, dims)
    h = rnd(x + rnd(o @ lw["wo"].T))
    b = rmsnorm(h, lw["ffn_norm"], dims.rms_eps)
    g = rnd(b @ lw["w_gate"].T)
    u = rnd(b @ lw["w_up"].T)
    f = rnd(silu(g) * u)
    out = rnd(h + rnd(f @ lw["w_down"].T))
    if return_kv:
        return out, k.reshape(T, nkv * d), v.reshape(T, nkv * d)
    return out


def lm_head(x: np.ndarray, weights: dict, dims: LLaDADims) -> np.ndarray:
    return rnd(rmsnorm(x, weights["final_norm"], dims.rms_eps) @ weights["lm_head"].T)


def dense_forward(tokens: np.ndarray, weights: dict, dims: LLaDADims) -> dict:
    """Plain (unfolded) forward of one sequence; returns per-layer inputs, K/V and logits."""
    T = tokens.shape[0]
    cos, sin = rope_tables(T, dims.head_dim, dims.rope_theta)
    x = weights["embed"][tokens]
    layer_in = [x]
    ks, vs = [], []
    for lw in weights["layers"]:
        x, k, v = block(x, lw, dims, cos, sin, return_kv=True)
        layer_in.append(x)
        ks.append(k)
        vs.append(v)
    return {
        "layer_in": np.stack(layer_in),
        "k": np.stack(ks),
        "v": np.stack(vs),
        "logits": lm_head(x, weights, dims),
    }
