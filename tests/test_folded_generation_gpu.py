"""folded_generate on the native pass against the reference (golden ``fgen.npz``).

``fgen.npz`` comes from the reference folded_generate
(actfold/speculative/folded_generation.py:44-238) over FoldedModel and the
restated tiny LLaDA block, 4 new tokens after a 24-id prompt:

* greedy: each step appends the argmax of the accepted sequence's last logits
  (every greedy choice of the fixture has a top-2 margin of at least 0.03,
  about four bf16 ulps of these logits, so the choice is defined);
* draft: AppendDraft proposes 3 one-id extensions per step, verified in one
  batched folded pass here (one forward each in the reference), and the
  greedy policy keeps the largest last-position logit (margins >= 0.05).

Compared: the accepted tokens after every step, each accepted node's stable
ratio (the mean over layers of its stable fraction; none on a step whose
parent was never run, as in the reference), the policy scores (within 2e-2,
the logits tolerance) and the final FoldedGenerationResult fields.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from actfold_b200 import workloads as W
from gen_inputs import TINY_FGEN, AppendDraft

pytestmark = pytest.mark.gpu


def _run(draft: bool):
    from actfold_b200.core import ActivationCache, FoldedModel, SimilarityGate
    from actfold_b200.llada import LLaDAModel
    from actfold_b200.speculative import GreedyAcceptancePolicy, folded_generate

    spec, dims = TINY_FGEN, W.LLADA_TINY
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    model = LLaDAModel.from_numpy(dims, w, device="cuda", max_pos=spec["T"] + spec["max_new_tokens"])
    fm = FoldedModel(model, ActivationCache(max_entries_per_layer=4096, device="cuda"), SimilarityGate(tau=spec["tau"]))
    steps, scores = [], []

    class Recording(GreedyAcceptancePolicy):
        def select(self, candidates, logits=None):
            scores.append([float(n.logits[:, -1, :].float().amax(dim=-1).mean()) for n in candidates])
            chosen = super().select(candidates, logits)
            steps.append((chosen.tokens[0].cpu().numpy(), float(chosen.metadata.get("stable_ratio", -1.0)),
                          np.stack([n.tokens[0].cpu().numpy() for n in candidates])))
            return chosen

    return steps, scores, fm, folded_generate, Recording(), dims, spec


@pytest.mark.parametrize("mode", ["greedy", "draft"])
def test_folded_generate_matches_reference(golden, mode):
    g = golden("fgen")
    steps, scores, fm, folded_generate, policy, dims, spec = _run(mode == "draft")
    prompt = torch.from_numpy(g["prompt"]).cuda()
    res = folded_generate(fm, prompt, spec["max_new_tokens"], folded_model=fm,
                          draft_generator=AppendDraft(dims.mask_id) if mode == "draft" else None,
                          acceptance_policy=policy, num_branches_per_step=spec["n_branches"] if mode == "draft" else 1)
    assert len(steps) == spec["max_new_tokens"]
    for i, (toks, ratio, cands) in enumerate(steps):
        np.testing.assert_array_equal(cands, g[f"{mode}/step{i}/candidates"])
        np.testing.assert_array_equal(toks, g[f"{mode}/step{i}/tokens"])
        assert abs(ratio - float(g[f"{mode}/step_ratio"][i])) <= 1e-6, (i, ratio)
    if mode == "draft":
        np.testing.assert_allclose(np.array(scores), g["draft/scores"], atol=2e-2)
    np.testing.assert_array_equal(res.tokens.cpu().numpy(), g[f"{mode}/tokens"])
    assert abs(res.stable_ratio - float(g[f"{mode}/stable_ratio"])) <= 1e-6
    assert res.num_folded_steps == int(g[f"{mode}/num_folded_steps"])
    assert res.final_branch_id == str(g[f"{mode}/final_branch_id"])
