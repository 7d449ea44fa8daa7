"""CPU timing of the reference's verification algorithm (TEST/BENCH INFRASTRUCTURE).

Used only by bench.py (cpu_baseline leg and the ``--impl reference`` arm).
The reference verifies a child by running its FULL layer on every row, then
gating and merging (actfold/core/folded_transformer.py:148-196): per child and
layer, a dense block recompute over all T rows + the cosine gate + the merge,
and the LM head over all rows. This module times that work with the oracle's
numpy restatement on the host cores, on a bounded sample, and extrapolates to
one full verification pass:

    t_pass = C * (L * (t_block + t_gate + t_merge) + t_lm_head)

Sample: one LLaDA block of the given dims on T rows (float32 numpy, BLAS on
all host threads), the gate and merge of that layer, and the LM head over a
vocabulary slice (scaled linearly to the full vocabulary).
"""

from __future__ import annotations

import os
import time

import numpy as np

from oracle import llada as L
from oracle.gate import gate
from oracle.numerics import round_bf16
from oracle.rows import merge


def _weights(dims: L.LLaDADims, rng: np.random.Generator) -> dict:
    H = dims.hidden
    q, kv = dims.n_heads * dims.head_dim, dims.n_kv_heads * dims.head_dim

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    return {
        "attn_norm": np.ones(H, np.float32), "wq": w(q, H), "wk": w(kv, H), "wv": w(kv, H), "wo": w(H, q),
        "ffn_norm": np.ones(H, np.float32), "w_gate": w(dims.ffn, H), "w_up": w(dims.ffn, H), "w_down": w(H, dims.ffn),
    }


class CpuSample:
    """Prepared inputs for repeated timing of the reference algorithm on the host."""

    def __init__(self, dims: L.LLaDADims, T: int, n_children: int, tau: float = 0.95, vocab_slice: int = 8192, seed: int = 0) -> None:
        rng = np.random.default_rng(seed)
        self.dims, self.T, self.C, self.tau = dims, T, n_children, tau
        self.lw = _weights(dims, rng)
        self.x = round_bf16(rng.standard_normal((T, dims.hidden), dtype=np.float32))
        self.parent_in = self.x.copy()
        self.parent_in[:16] += np.float32(0.5) * rng.standard_normal((16, dims.hidden), dtype=np.float32)
        self.parent_out = rng.standard_normal((T, dims.hidden), dtype=np.float32)
        self.vs = min(vocab_slice, dims.vocab)
        self.lm = (rng.standard_normal((self.vs, dims.hidden), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        self.cos, self.sin = L.rope_tables(T, dims.head_dim, dims.rope_theta)
        self.threads = os.cpu_count() or 1

    def time_pass(self) -> tuple[float, dict]:
        """Seconds of one full verification pass (extrapolated) and the measured parts."""
        t0 = time.perf_counter()
        out = L.block(self.x, self.lw, self.dims, self.cos, self.sin)
        t1 = time.perf_counter()
        g = gate(self.x[None], self.parent_in[None], self.tau, "cosine", 1e-8, "f32")
        t2 = time.perf_counter()
        merge(self.parent_out[None], out[None], g.mask)
        t3 = time.perf_counter()
        _ = self.x @ self.lm.T
        t4 = time.perf_counter()
        t_block, t_gate, t_merge = t1 - t0, t2 - t1, t3 - t2
        t_lm = (t4 - t3) * (self.dims.vocab / self.vs)
        per_pass = self.C * (self.dims.n_layers * (t_block + t_gate + t_merge) + t_lm)
        return per_pass, {"block_s": t_block, "gate_s": t_gate, "merge_s": t_merge, "lm_head_s": t_lm, "sample_s": t4 - t0}
