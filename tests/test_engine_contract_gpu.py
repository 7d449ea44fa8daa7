"""The verification engine against the reference engine's contract (golden ``engine.npz``).

``engine.npz`` comes from the reference's ActFoldVerificationEngine.verify_branch
(actfold/speculative/verification_engine.py:75-144) over FoldedModel and the
restated tiny LLaDA block: 4 children of one parent (2, 4, 6 and 8 unmasked
positions), verified at acceptance thresholds 0 and 0.890625, then two
grandchildren verified with ``verify_branch(accepted child, grandchild)``.

Compared per child: the acceptance decision (``stable_ratio >= threshold``),
the stable ratio (mean over layers of the per-layer stable fraction) and
``metadata["stable_ratio"]``, the per-layer ratios of the child's
StabilityProfile, ``metadata["actfold_score"]`` (the mean of the child's
logits; within 2e-2 of the logits' scale, the logits tolerance), and that a
rejected child's cache entries are cleared while an accepted child keeps them.
The batched ``verify_branches`` must give the same results as one
``verify_branch`` call per child.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from actfold_b200 import workloads as W
from gen_inputs import TINY_ENGINE, engine_children

pytestmark = pytest.mark.gpu

RATIO_TOL = 1e-6
SCORE_TOL = 2e-2  # of the largest |logit| of the child


@pytest.fixture(scope="module")
def setup(golden):
    from actfold_b200.llada import LLaDAModel

    g = golden("engine")
    dims, spec = W.LLADA_TINY, TINY_ENGINE
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    parent, _ = W.llada_tokens(spec["T"], spec["n_prompt"], spec["mask_frac"], 1, 1, dims.mask_id, spec["token_seed"])
    children = engine_children(parent, dims.mask_id, spec)
    np.testing.assert_array_equal(parent, g["parent"])
    np.testing.assert_array_equal(children, g["children"])
    model = LLaDAModel.from_numpy(dims, w, device="cuda", max_pos=spec["T"])
    return dict(g=g, dims=dims, spec=spec, model=model, parent=parent, children=children)


def _engine(s, threshold):
    from actfold_b200.core import ActivationCache, SimilarityGate
    from actfold_b200.speculative import ActFoldVerificationEngine

    cache = ActivationCache(max_entries_per_layer=8 * s["spec"]["T"], device="cuda")
    # Each child holds cache entries before it is verified; a rejection must clear them.
    for c in range(s["children"].shape[0]):
        cache.put(f"child{c}", 0, {"hidden_states": torch.zeros(1, s["spec"]["T"], 8, device="cuda")})
    eng = ActFoldVerificationEngine(s["model"], cache=cache, gate=SimilarityGate(s["spec"]["tau"]),
                                    acceptance_threshold=threshold)
    return eng, cache


def _has_entries(cache, branch_id) -> bool:
    return cache.has_entry(branch_id, 0)


def _logit_scale(eng, pb, tokens) -> float:
    res = eng.verify_tokens(pb, torch.from_numpy(np.ascontiguousarray(tokens[None])).pin_memory())
    return float(res["logits"].float().abs().max())


@pytest.mark.parametrize("name", ["t0", "t1"])
def test_verify_branch_matches_reference_engine(setup, name):
    from actfold_b200.profiler import GLOBAL_STABILITY_PROFILER
    from actfold_b200.speculative import Branch

    s, g = setup, setup["g"]
    thr = float(g[f"{name}/threshold"])
    eng, cache = _engine(s, thr)
    pb = Branch("parent", None, torch.from_numpy(s["parent"])[None])
    for c in range(s["children"].shape[0]):
        tokens = torch.from_numpy(s["children"][c])[None]
        cb = Branch(f"child{c}", "parent", tokens)
        r = eng.verify_branch(pb, cb)
        assert r.accepted == bool(g[f"{name}/accepted"][c]) == cb.accepted
        assert abs(r.stable_ratio - float(g[f"{name}/ratio"][c])) <= RATIO_TOL
        assert cb.metadata["stable_ratio"] == r.stable_ratio
        prof = GLOBAL_STABILITY_PROFILER.get_profile(cb.branch_id)
        assert r.stability_profile is prof
        np.testing.assert_allclose([st.stable_ratio for st in prof.layer_stats], g[f"{name}/layer_ratio"][c], atol=RATIO_TOL)
        assert _has_entries(cache, cb.branch_id) == bool(g[f"{name}/cached"][c])
        scale = _logit_scale(eng, pb, s["children"][c])
        assert abs(cb.metadata["actfold_score"] - float(g[f"{name}/score"][c])) <= SCORE_TOL * scale


def test_verify_branches_batch_equals_single_calls(setup):
    from actfold_b200.speculative import Branch

    s, g = setup, setup["g"]
    thr = float(g["t1/threshold"])
    eng, cache = _engine(s, thr)
    pb = Branch("parent", None, torch.from_numpy(s["parent"])[None])
    kids = [Branch(f"child{c}", "parent", torch.from_numpy(s["children"][c])[None]) for c in range(s["children"].shape[0])]
    batch = eng.verify_branches(pb, kids)
    eng2, _ = _engine(s, thr)
    for c, rb in enumerate(batch):
        single = eng2.verify_branch(pb, Branch(f"child{c}", "parent", torch.from_numpy(s["children"][c])[None]))
        assert rb.accepted == single.accepted == bool(g["t1/accepted"][c])
        assert rb.stable_ratio == single.stable_ratio
        # A batch and a single child run GEMMs of different token tiles (a
        # 16-token tile on one CTA, a wider one on a CTA pair), whose fp32
        # sums may round a few logits differently: scores agree to 1e-3 of
        # the logits' scale.
        scale = _logit_scale(eng2, pb, s["children"][c])
        assert abs(rb.child_branch.metadata["actfold_score"] - single.child_branch.metadata["actfold_score"]) <= 1e-3 * scale
        assert _has_entries(cache, f"child{c}") == bool(g["t1/cached"][c])


def test_chained_verify_branch_against_an_accepted_child(setup):
    """verify_branch(child, grandchild): the child's tokens are the parent now (the reference re-runs its dense pass)."""
    from actfold_b200.profiler import GLOBAL_STABILITY_PROFILER
    from actfold_b200.speculative import Branch

    s, g = setup, setup["g"]
    eng, _ = _engine(s, 0.0)
    pb = Branch("parent", None, torch.from_numpy(s["parent"])[None])
    k = int(g["grand/child"])
    kb = Branch(f"child{k}", "parent", torch.from_numpy(s["children"][k])[None])
    assert eng.verify_branch(pb, kb).accepted
    grand = g["grand/tokens"]
    for i in range(grand.shape[0]):
        gb = Branch(f"grand{i}", kb.branch_id, torch.from_numpy(grand[i])[None])
        r = eng.verify_branch(kb, gb)
        assert abs(r.stable_ratio - float(g["grand/ratio"][i])) <= RATIO_TOL
        prof = GLOBAL_STABILITY_PROFILER.get_profile(gb.branch_id)
        np.testing.assert_allclose([st.stable_ratio for st in prof.layer_stats], g["grand/layer_ratio"][i], atol=RATIO_TOL)
        scale = _logit_scale(eng, kb, grand[i])
        assert abs(gb.metadata["actfold_score"] - float(g["grand/score"][i])) <= SCORE_TOL * scale
