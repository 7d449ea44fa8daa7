"""The headline folded pass at full LLaDA-8B size (8 children x 1024 tokens, d = 16, tau 0.95).

Checked in full by ``fullsize_util.check_folded_pass``: gate decisions at
every layer against ``SimilarityGate``, stable rows bit-identical to the
parent's, the divergent rows of all 32 layers' outputs for all 8 children and
of the final logits against the fp32 restatement of the block and of the LM
head (relative error <= 2e-2, cosine >= 0.999, argmax agreement >= 99.9 %).
"""

from __future__ import annotations

import pytest
import torch

from actfold_b200 import workloads as W
from fullsize_util import check_folded_pass

pytestmark = pytest.mark.gpu

TAU = 0.95


def test_headline_pass_every_layer_every_child():
    from actfold_b200.llada import LLaDAModel

    dims = W.LLADA_8B
    model = LLaDAModel.random(dims, seed=1234, device="cuda", max_pos=1024)
    parent, _ = W.llada_tokens(1024, 256, 0.5, 1, 1, dims.mask_id, seed=42)
    children = W.llada_children(parent, 8, 16, dims.mask_id, seed=1000)
    pc = model.parent_pass(torch.from_numpy(parent).cuda(), tau=TAU)
    logits, plan = model.verify(torch.from_numpy(children).cuda(), pc, TAU)
    torch.cuda.synchronize()
    plan.check_status()
    st = check_folded_pass(model, pc, parent, children, TAU, logits, plan)
    print(f"llada8b T=1024 d=16: {st}")
