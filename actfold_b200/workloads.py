"""Seeded synthetic workloads for the folded verification path.

No datasets or checkpoints are involved: every weight and token id below is
drawn from a seeded numpy PCG64 generator (or, for the full-size LLaDA weights,
a seeded CUDA generator), with the shapes and distributions of the workloads:

* demo      -- demo.py's synthetic Transformer (4 post-norm layers, hidden 128,
               8 heads, FFN 512 GELU, vocab 1000); parent of 16 uniform ids,
               children that replace one random position with a fresh id
               (demo.py:408-477, draft_generator.py:94-107).
* llada-8b  -- LLaDA-8B architecture: 32 layers, hidden 4096, 32 heads x 128,
               SwiGLU 12288, RMSNorm 1e-5, RoPE theta 5e5, vocab 126464,
               mask id 126336.
* dream-7b  -- Qwen2.5-7B layout: 28 layers, hidden 3584, 28 q / 4 kv heads,
               SwiGLU 18944, RMSNorm 1e-6, RoPE 1e6, vocab 152064, mask 151666.

Token layout of the LLaDA workloads: a prompt of uniform ids in
[0, mask_id), then generation positions of which a seeded fraction holds the
mask id (the rest uniform ids); each child unmasks ``d`` of the parent's
masked positions (chosen uniformly) to uniform ids in [0, mask_id).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ModelDims:
    """Architecture of an LLaDA/Dream-style block stack."""

    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rms_eps: float = 1e-5
    rope_theta: float = 500000.0
    mask_id: int = 126336

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def params_per_layer(self) -> int:
        H = self.hidden
        return H * self.q_dim + 2 * H * self.kv_dim + self.q_dim * H + 3 * H * self.ffn


LLADA_8B = ModelDims(32, 4096, 32, 32, 128, 12288, 126464, 1e-5, 500000.0, 126336)
DREAM_7B = ModelDims(28, 3584, 28, 4, 128, 18944, 152064, 1e-6, 1000000.0, 151666)
# A reduced LLaDA-shaped model for parity tests the oracle finishes in seconds.
LLADA_TINY = ModelDims(2, 256, 2, 2, 128, 512, 512, 1e-5, 500000.0, 500)
# Reduced GQA (Dream-shaped) model for parity tests.
DREAM_TINY = ModelDims(2, 256, 2, 1, 128, 384, 512, 1e-6, 1000000.0, 500)

DIMS = {"llada-8b": LLADA_8B, "dream-7b": DREAM_7B, "llada-tiny": LLADA_TINY, "dream-tiny": DREAM_TINY}


def round_bf16_np(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16-representable float32 (ties to even)."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + (((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF))) & np.uint64(0xFFFF0000)).astype(np.uint32)
    return r.view(np.float32).reshape(a.shape)


def llada_weights_numpy(dims: ModelDims, seed: int = 0, std: float = 0.02) -> dict:
    """bf16-representable float32 weights, N(0, std) for every matrix, ones for norms."""
    rng = np.random.default_rng(seed)

    def w(*shape):
        return round_bf16_np(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    H = dims.hidden
    layers = []
    for _ in range(dims.n_layers):
        layers.append(
            {
                "attn_norm": np.ones(H, np.float32),
                "wq": w(dims.q_dim, H),
                "wk": w(dims.kv_dim, H),
                "wv": w(dims.kv_dim, H),
                "wo": w(H, dims.q_dim),
                "ffn_norm": np.ones(H, np.float32),
                "w_gate": w(dims.ffn, H),
                "w_up": w(dims.ffn, H),
                "w_down": w(H, dims.ffn),
            }
        )
    return {
        "embed": w(dims.vocab, H),
        "layers": layers,
        "final_norm": np.ones(H, np.float32),
        "lm_head": w(dims.vocab, H),
    }


def llada_tokens(
    T: int,
    n_prompt: int,
    mask_frac: float,
    n_children: int,
    d: int,
    mask_id: int,
    seed: int = 42,
) -> tuple[np.ndarray, np.ndarray]:
    """Parent ids [T] and children ids [C, T] (int64) for an LLaDA-style workload."""
    rng = np.random.default_rng(seed)
    parent = rng.integers(0, mask_id, size=T, dtype=np.int64)
    gen = np.arange(n_prompt, T)
    n_mask = int(round(mask_frac * gen.size))
    masked = np.sort(rng.choice(gen, size=n_mask, replace=False))
    parent[masked] = mask_id
    return parent, _unmask_children(parent, masked, n_children, d, mask_id, rng)


def _unmask_children(parent: np.ndarray, masked: np.ndarray, n_children: int, d: int, mask_id: int, rng) -> np.ndarray:
    children = np.repeat(parent[None], n_children, axis=0)
    if d > masked.size:
        raise ValueError(f"d={d} exceeds the {masked.size} masked positions")
    for c in range(n_children):
        pos = rng.choice(masked, size=d, replace=False)
        children[c, pos] = rng.integers(0, mask_id, size=d, dtype=np.int64)
    return children


def llada_children(parent: np.ndarray, n_children: int, d: int, mask_id: int, seed: int) -> np.ndarray:
    """Children [C, T] of an existing parent: each unmasks d of its masked positions (seeded)."""
    rng = np.random.default_rng(seed)
    masked = np.nonzero(parent == mask_id)[0]
    return _unmask_children(parent, masked, n_children, d, mask_id, rng)


def uniform_edit_children(parent: np.ndarray, n_children: int, d: int, id_hi: int, seed: int) -> np.ndarray:
    """Children [C, T] that each differ from the parent at ``d`` uniformly chosen positions.

    The new ids are uniform over [0, id_hi) and never equal the parent's id at
    that position (the Dream-7B workload: 16 children, 8 positions each).
    """
    rng = np.random.default_rng(seed)
    T = parent.shape[0]
    if d > T:
        raise ValueError(f"d={d} exceeds the sequence length {T}")
    children = np.repeat(parent[None], n_children, axis=0)
    for c in range(n_children):
        for p in rng.choice(T, size=d, replace=False):
            new = parent[p]
            while new == parent[p]:
                new = int(rng.integers(0, id_hi))
            children[c, p] = new
    return children


def demo_weights(seed: int = 42, vocab: int = 1000, hidden: int = 128, n_layers: int = 4, std: float = 0.02) -> dict:
    """Weights of demo.py's SyntheticTransformer re-drawn N(0, std); zero biases, unit LayerNorms."""
    rng = np.random.default_rng(seed)

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    H = hidden
    layers = []
    for _ in range(n_layers):
        layers.append(
            {
                "in_proj_weight": w(3 * H, H),
                "in_proj_bias": np.zeros(3 * H, np.float32),
                "out_proj_weight": w(H, H),
                "out_proj_bias": np.zeros(H, np.float32),
                "norm1_weight": np.ones(H, np.float32),
                "norm1_bias": np.zeros(H, np.float32),
                "ffn0_weight": w(4 * H, H),
                "ffn0_bias": np.zeros(4 * H, np.float32),
                "ffn2_weight": w(H, 4 * H),
                "ffn2_bias": np.zeros(H, np.float32),
                "norm2_weight": np.ones(H, np.float32),
                "norm2_bias": np.zeros(H, np.float32),
            }
        )
    return {"embedding": w(vocab, H), "layers": layers, "lm_head": w(vocab, H)}


def demo_tokens(seed: int = 42, T: int = 16, n_children: int = 2, vocab: int = 1000) -> tuple[np.ndarray, np.ndarray]:
    """Parent ids [T] and children [C, T], each child replacing max(1, int(0.05 T)) positions."""
    rng = np.random.default_rng(seed)
    parent = rng.integers(0, vocab, size=T, dtype=np.int64)
    n_flip = max(1, int(T * 0.05))
    children = np.repeat(parent[None], n_children, axis=0)
    for c in range(n_children):
        pos = rng.choice(T, size=n_flip, replace=False)
        for p in pos:
            new = parent[p]
            while new == parent[p]:
                new = int(rng.integers(0, vocab))
            children[c, p] = new
    return parent, children
