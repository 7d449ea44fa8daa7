"""Full-size folded passes of the two model families the path serves, checked in full.

* LLaDA-8B architecture, 8 children of a 512-id parent (128 prompt ids, half
  of the other 384 the mask id), each child unmasking d in {4, 16, 64}
  positions, tau 0.95: every layer and every child.
* Dream-7B architecture (Qwen2.5-7B layout, GQA with 4 KV heads, FFN 18944),
  16 children of a 1024-id parent (256 prompt ids, 75 % of the generation
  positions masked), each differing from the parent at 8 uniformly chosen
  positions, tau swept over {0.90, 0.95, 0.98} (bf16(0.98) = 0.98046875 moves
  the gate's decision boundary): every layer and every child.

What is checked, and the tolerances, are those of ``fullsize_util``: gate
decisions against ``SimilarityGate`` at every layer, stable rows bit-identical
to the parent's, divergent rows of every layer's output and of the final
logits against the fp32 restatement (relative error <= 2e-2, cosine >=
0.999, argmax agreement >= 99.9 %).
"""

from __future__ import annotations

import gc

import pytest
import torch

from actfold_b200 import workloads as W
from fullsize_util import check_folded_pass

pytestmark = pytest.mark.gpu


def _release():
    gc.collect()
    torch.cuda.empty_cache()


@pytest.fixture(scope="module")
def llada_512():
    from actfold_b200.llada import LLaDAModel

    dims = W.LLADA_8B
    model = LLaDAModel.random(dims, seed=1234, device="cuda", max_pos=512)
    parent, _ = W.llada_tokens(512, 128, 0.5, 1, 1, dims.mask_id, seed=42)
    pc = model.parent_pass(torch.from_numpy(parent).cuda(), tau=0.95)
    yield model, parent, pc
    del model, pc
    _release()


@pytest.mark.parametrize("d", [4, 16, 64])
def test_llada8b_512_tokens_8_children(llada_512, d):
    model, parent, pc = llada_512
    children = W.llada_children(parent, 8, d, model.dims.mask_id, seed=2000 + d)
    logits, plan = model.verify(torch.from_numpy(children).cuda(), pc, 0.95)
    torch.cuda.synchronize()
    plan.check_status()
    st = check_folded_pass(model, pc, parent, children, 0.95, logits, plan)
    print(f"llada8b T=512 d={d}: {st}")


@pytest.fixture(scope="module")
def dream_1024():
    from actfold_b200.llada import LLaDAModel

    dims = W.DREAM_7B
    model = LLaDAModel.random(dims, seed=4321, device="cuda", max_pos=1024)
    parent, _ = W.llada_tokens(1024, 256, 0.75, 1, 1, dims.mask_id, seed=42)
    children = W.uniform_edit_children(parent, 16, 8, dims.mask_id, seed=3000)
    yield model, parent, children
    del model
    _release()


@pytest.mark.parametrize("tau", [0.90, 0.95, 0.98])
def test_dream7b_1024_tokens_16_children_tau_sweep(dream_1024, tau):
    model, parent, children = dream_1024
    pc = model.parent_pass(torch.from_numpy(parent).cuda(), tau=tau)
    logits, plan = model.verify(torch.from_numpy(children).cuda(), pc, tau)
    torch.cuda.synchronize()
    plan.check_status()
    st = check_folded_pass(model, pc, parent, children, tau, logits, plan)
    print(f"dream7b T=1024 tau={tau}: {st}")
