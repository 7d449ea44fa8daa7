"""FoldedModel with a FoldingScheduler on the native pass, against the reference (golden ``sched.npz``).

``sched.npz`` comes from the reference FoldedModel with
FoldingScheduler(base_tau=0.95, num_layers=4, num_steps=4, disabled_layers={1})
over the restated 4-layer tiny LLaDA block (actfold/core/folded_transformer.py:
107-119): at steps 0 and 2 layers 0 and 2 fold, each at its own
``get_tau(layer, step)``, layer 1 (disabled) and layer 3 (the final layer)
recompute every row; at step 3 (the final step) no layer folds.

Checked per step, for the batched native pass of all 4 children:
* the folded layers and the tau each used (the StabilityProfile's layer_stats);
* the stable masks of the folded layers: bit-exact except on rows whose f32
  similarity (on the oracle's rows) lies within SCHED_WINDOW = 1e-2 of the bf16
  decision boundary -- after a layer that does not fold every row is
  recomputed, so two correct recomputations that round differently can decide
  such rows either way (measured up to 4.5e-3 apart between numpy and torch);
* the logits of every row whose masks agree: relative error <= 2e-2 of the
  scale, cosine >= 0.999;
* the gate's tau after the step (the reference leaves the shared gate at the
  last folded layer's tau).
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np
import pytest
import torch

from actfold_b200 import workloads as W
from gen_inputs import TINY_SCHED
from oracle import folding as OF
from oracle import llada as OL
from oracle.gate import exempt_rows, gate
from oracle.numerics import from_bf16_bits

pytestmark = pytest.mark.gpu

SCHED_WINDOW = 1e-2


def test_folded_model_with_scheduler_matches_reference(golden):
    from actfold_b200.core import ActivationCache, FoldedModel, FoldingScheduler, SimilarityGate
    from actfold_b200.llada import LLaDAModel
    from actfold_b200.profiler import GLOBAL_STABILITY_PROFILER

    g = golden("sched")
    spec = TINY_SCHED
    dims = dataclasses.replace(W.LLADA_TINY, n_layers=spec["n_layers"])
    od = OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab,
                      dims.rms_eps, dims.rope_theta)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    parent, children = W.llada_tokens(spec["T"], spec["n_prompt"], spec["mask_frac"], spec["n_children"], spec["d"],
                                      dims.mask_id, spec["token_seed"])
    np.testing.assert_array_equal(children, g["children"])
    C = children.shape[0]
    model = LLaDAModel.from_numpy(dims, w, device="cuda", max_pos=spec["T"])
    sched = FoldingScheduler(base_tau=spec["tau"], num_layers=dims.n_layers, num_steps=spec["num_steps"],
                             disabled_layers=set(spec["disabled_layers"]))
    gate_mod = SimilarityGate(tau=spec["tau"])
    fm = FoldedModel(model, ActivationCache(max_entries_per_layer=4096, device="cuda"), gate_mod, scheduler=sched)
    fm(torch.from_numpy(parent)[None].cuda(), branch_id="parent")
    par = OF.llada_parent(parent, w, od)
    for step in spec["steps"]:
        ids = [f"s{step}c{c}" for c in range(C)]
        for b in ids:
            GLOBAL_STABILITY_PROFILER.reset_branch(b)
        logits = fm(torch.from_numpy(children).cuda(), branch_id=ids, parent_branch_id="parent", step_idx=step)
        got = logits.float().cpu().numpy()
        layers = list(g[f"step{step}/layers"])
        folds = [sched.should_fold(li, step) for li in range(dims.n_layers)]
        taus = [sched.get_tau(li, step) if folds[li] else spec["tau"] for li in range(dims.n_layers)]
        ora = OF.llada_folded_children(children, par, w, od, spec["tau"], taus, folds)
        ok_rows = np.ones(children.shape, bool)
        for c, b in enumerate(ids):
            prof = GLOBAL_STABILITY_PROFILER.get_profile(b)
            stats = prof.layer_stats if prof is not None else []
            assert [st.layer_idx for st in stats] == layers, (step, c)
            np.testing.assert_allclose([st.tau_used for st in stats], g[f"step{step}/taus"], rtol=0, atol=1e-12)
            for i, (st, li) in enumerate(zip(stats, layers)):
                m = np.ones(spec["T"], bool)
                if st.divergence_positions is not None:
                    m[st.divergence_positions[:, 1].cpu().numpy()] = False
                ref = g[f"step{step}/masks"][i, c]
                r = gate(ora["states"][li][c][None], par["layer_in"][li][None], taus[li], "cosine", 1e-8, "bf16")
                exempt = exempt_rows(r, SCHED_WINDOW if li > 0 else 1e-4)[0]
                mism = m != ref
                assert not (mism & ~exempt).any(), (step, li, c, np.nonzero(mism & ~exempt))
                ok_rows[c] &= ~mism
        ref = from_bf16_bits(g[f"step{step}/logits_bits"])
        a, b = got[ok_rows].astype(np.float64), ref[ok_rows].astype(np.float64)
        rel = float(np.abs(a - b).max() / np.abs(b).max())
        cos = float((a * b).sum() / math.sqrt((a * a).sum() * (b * b).sum()))
        assert rel <= 2e-2 and cos >= 0.999, (step, rel, cos)
        assert gate_mod.tau == pytest.approx(float(g[f"step{step}/gate_tau_after"]), abs=1e-12)
