"""Candidate-key window of the folded pass's attention (many children) against the oracle.

With a bound on any child's candidate rows, each tile of 128 packed query rows
scans only the candidate key blocks around its own rows (the candidate list is
ordered by child). Here 64 children x 7 edited tokens give 448 candidate rows
(four candidate blocks, a window of three, shifted at both ends) and 96 x 7
give six blocks; 7 does not divide 128, so children straddle tile edges. Results must match the oracle (masks exact,
bf16 tolerance for logits) and the unwindowed pass within the same tolerance;
a bound below the real per-child count must be reported, not ignored.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from actfold_b200 import workloads as W
from oracle import folding as OF
from test_native_gpu import _argmax_agreement, _cos, _odims, _rel

pytestmark = pytest.mark.gpu

DIMS = W.LLADA_TINY


@pytest.fixture(scope="module")
def setup():
    from actfold_b200.llada import LLaDAModel

    w = W.llada_weights_numpy(DIMS, seed=7)
    parent, _ = W.llada_tokens(64, 8, 0.75, 1, 1, DIMS.mask_id, seed=21)
    model = LLaDAModel.from_numpy(DIMS, w, device="cuda", max_pos=64)
    return dict(w=w, parent=parent, model=model, pc=model.parent_pass(torch.from_numpy(parent).cuda(), tau=0.95))


@pytest.mark.parametrize("n_children", [64, 96])
def test_windowed_attention_matches_oracle(setup, n_children):
    m, pc = setup["model"], setup["pc"]
    children = W.llada_children(setup["parent"], n_children, 7, DIMS.mask_id, seed=100 + n_children)
    ct = torch.from_numpy(children).cuda()
    logits, plan = m.verify(ct, pc, 0.95)
    assert plan.child_cap == 7 and plan.m_cap == n_children * 7
    torch.cuda.synchronize()
    plan.check_status()
    masks = plan.stable_masks().cpu().numpy()
    got = logits.float().cpu().numpy()
    od = _odims(DIMS)
    ref = OF.llada_folded_children(children, OF.llada_parent(setup["parent"], setup["w"], od), setup["w"], od, 0.95)
    np.testing.assert_array_equal(masks, ref["masks"])
    assert _rel(got, ref["logits"]) <= 2e-2
    assert _cos(got, ref["logits"]) >= 0.999
    assert _argmax_agreement(got, ref["logits"]) >= 0.999
    # the same pass scanning every candidate block
    plan.set_child_cap(0)
    full = torch.empty_like(logits)
    plan.run(ct, full)
    torch.cuda.synchronize()
    plan.check_status()
    np.testing.assert_array_equal(plan.stable_masks().cpu().numpy(), masks)
    assert _rel(got, full.float().cpu().numpy()) <= 2e-2


def test_bound_below_the_real_count_is_reported(setup):
    m, pc = setup["model"], setup["pc"]
    children = W.llada_children(setup["parent"], 64, 7, DIMS.mask_id, seed=7)
    ct = torch.from_numpy(children).cuda()
    _, plan = m.verify(ct, pc, 0.95)
    plan.set_child_cap(1)  # window of one block: the children at tile edges have keys outside it
    out = torch.empty((64, 64, DIMS.vocab), dtype=torch.bfloat16, device="cuda")
    plan.run(ct, out)
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        plan.check_status()
    plan.set_child_cap(7)
    plan.run(ct, out)
    torch.cuda.synchronize()
    plan.check_status()
