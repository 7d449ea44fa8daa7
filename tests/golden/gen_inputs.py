"""Deterministic inputs shared by the golden-vector generator and the tests.

Everything is drawn from numpy's PCG64 generator, so the same seed gives the
same bits here and on any other machine with the same numpy.
"""

from __future__ import annotations

import hashlib

import numpy as np

from oracle.numerics import round_to

# (name, seed, B, T, H, dtype, tau, metric)
GATE_CASES = [
    ("bf16_cos_t095", 1, 4, 256, 1024, "bf16", 0.95, "cosine"),
    ("bf16_cos_t090", 2, 4, 256, 1024, "bf16", 0.90, "cosine"),
    ("bf16_cos_t098", 3, 4, 256, 1024, "bf16", 0.98, "cosine"),
    ("bf16_cos_h4096", 4, 2, 128, 4096, "bf16", 0.95, "cosine"),
    ("bf16_cos_h3584", 5, 2, 64, 3584, "bf16", 0.95, "cosine"),
    ("f32_cos_t095", 6, 4, 256, 512, "f32", 0.95, "cosine"),
    ("f16_cos_t095", 7, 2, 256, 1024, "f16", 0.95, "cosine"),
    ("bf16_l2_t050", 8, 2, 128, 256, "bf16", 0.5, "l2"),
    ("bf16_pearson_t095", 9, 2, 128, 1024, "bf16", 0.95, "pearson"),
    ("f32_l2_t050", 10, 2, 128, 256, "f32", 0.5, "l2"),
    ("f32_pearson_t095", 11, 2, 128, 512, "f32", 0.95, "pearson"),
]


def gate_inputs(seed: int, B: int, T: int, H: int, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """Parent/child rows whose cosine spreads over [0.85, 1] plus edge rows.

    Row (0,0) identical, (0,1) both zero, (0,2) negated, (0,3) child zero,
    (0,4) tiny-magnitude copy, (0,5) large-magnitude rows.
    """
    rng = np.random.default_rng(seed)
    parent = rng.standard_normal((B, T, H), dtype=np.float32)
    noise = rng.standard_normal((B, T, H), dtype=np.float32)
    target = rng.uniform(0.85, 1.0, size=(B, T, 1)).astype(np.float32)
    s = np.sqrt(1.0 / (target * target) - 1.0).astype(np.float32)
    child = parent + s * noise
    child[0, 0] = parent[0, 0]
    child[0, 1] = 0.0
    parent[0, 1] = 0.0
    child[0, 2] = -parent[0, 2]
    child[0, 3] = 0.0
    child[0, 4] = parent[0, 4] * np.float32(1e-3)
    parent[0, 5] *= np.float32(64.0)
    child[0, 5] = parent[0, 5] + np.float32(8.0) * noise[0, 5]
    return round_to(child, dtype), round_to(parent, dtype)


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


# Tiny LLaDA-shaped folded workload: dims, token layout and tau.
TINY_LLADA = dict(T=64, n_prompt=16, mask_frac=0.5, n_children=4, d=4, tau=0.95, weight_seed=7, token_seed=42)
# Chained folding: grandchildren of child `chain_child` of the TINY_LLADA workload.
TINY_LLADA_CHAIN = dict(TINY_LLADA, chain_child=1, chain_n=3, chain_d=3, chain_seed=44)
# Children of another length than their parent: a 48-id parent, children of 64 ids
# (16 appended) and of 40 ids (a prefix with d edits).
TINY_LLADA_RESIZE = dict(TINY_LLADA, parent_len=48, short_len=40, n_children=3, d=2)
TINY_DREAM = dict(T=64, n_prompt=16, mask_frac=0.75, n_children=3, d=3, tau=0.95, weight_seed=11, token_seed=43)
DEMO = dict(T=16, n_children=2, tau=0.95, weight_seed=42, token_seed=42)
# Verification-engine contract: the TINY_LLADA workload (4 children) verified at
# two acceptance thresholds (0 and one between the children's stable ratios),
# then grandchildren of an accepted child verified against it.
# Child c unmasks child_d[c] positions, so the children's stable ratios differ.
TINY_ENGINE = dict(TINY_LLADA, child_d=(2, 4, 6, 8), chain_n=2, chain_d=2, chain_seed=45)


def engine_children(parent, mask_id: int, spec: dict):
    """Children [C, T] of the engine workload: child c unmasks spec["child_d"][c] positions."""
    from actfold_b200 import workloads as W

    return np.concatenate([W.llada_children(parent, 1, d, mask_id, spec["token_seed"] + 100 + c)
                           for c, d in enumerate(spec["child_d"])])
# FoldingScheduler over a 4-layer tiny LLaDA: base tau 0.95, 4 diffusion steps,
# layer 1 disabled; children verified at steps 0, 2 and 3 (the final step folds nothing).
TINY_SCHED = dict(TINY_LLADA, n_layers=4, num_steps=4, disabled_layers=(1,), steps=(0, 2, 3))
# folded_generate over the tiny LLaDA block: a 24-id prompt, 4 new tokens,
# greedy single-candidate steps, then 3 drafted candidates per step chosen by
# the greedy policy. The prompt seed is the first from prompt_seed on whose
# every greedy choice has a top-2 logit margin of at least min_margin.
TINY_FGEN = dict(T=24, max_new_tokens=4, n_branches=3, weight_seed=7, prompt_seed=50, min_margin=0.03, tau=0.95)


class AppendDraft:
    """Deterministic drafts for folded_generate: each candidate appends one id drawn from a seeded PCG64 stream.

    ``generate(parent, num_branches, seed, max_new_tokens)`` follows the
    reference DraftGenerator's call; only ``.tokens`` of the returned objects
    is read.
    """

    def __init__(self, id_hi: int, base_seed: int = 777) -> None:
        self.id_hi, self.base_seed = id_hi, base_seed

    def generate(self, parent, num_branches: int = 2, seed=None, max_new_tokens: int = 0):
        import types

        import torch

        rng = np.random.default_rng(self.base_seed + (seed or 0))
        out = []
        for _ in range(num_branches):
            new = torch.from_numpy(rng.integers(0, self.id_hi, size=(parent.tokens.shape[0], max_new_tokens)))
            out.append(types.SimpleNamespace(tokens=torch.cat([parent.tokens, new.to(parent.tokens.device, parent.tokens.dtype)], dim=1)))
        return out
