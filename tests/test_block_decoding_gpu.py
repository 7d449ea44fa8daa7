"""Block decoding with folded verification steps (the LLaDA-8B block-decoding workload, tiny) vs the oracle.

Each step folds C children of the current block against the current parent
and promotes the accepted one in place; the oracle (oracle/block_decoding.py)
folds the same children with the reference's semantics and promotes by the
reference's rule (a verified child's merged states become the parent). The
trajectory (accepted child and unmasked count per step, final canvas) must be
identical; the final parent's states and logits within the bf16 tolerance
(max relative error <= 2e-2, cosine >= 0.999).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from actfold_b200 import workloads as W
from oracle import block_decoding as OB
from test_native_gpu import _cos, _odims, _rel

pytestmark = pytest.mark.gpu

DIMS = W.LLADA_TINY


@pytest.fixture(scope="module")
def model_and_weights():
    from actfold_b200.llada import LLaDAModel

    w = W.llada_weights_numpy(DIMS, seed=7)
    return LLaDAModel.from_numpy(DIMS, w, device="cuda", max_pos=64), w


@pytest.mark.parametrize("acceptance_threshold,use_graph", [(0.0, True), (0.95, False)])
def test_block_decoding_matches_oracle(model_and_weights, acceptance_threshold, use_graph):
    from actfold_b200.speculative import BlockDecoder, BlockDecodingConfig, SyntheticDraft

    model, w = model_and_weights
    cfg = BlockDecodingConfig(prompt_len=32, gen_len=32, block_size=16, n_children=4, min_edits=2, max_edits=4,
                              threshold=0.9, tau=0.95, acceptance_threshold=acceptance_threshold, seed=5)
    prompt = np.random.default_rng(3).integers(0, DIMS.mask_id, size=cfg.prompt_len, dtype=np.int64)
    draft = SyntheticDraft(DIMS.mask_id, seed=cfg.seed)
    res = BlockDecoder(model, cfg, draft, use_graph=use_graph).run(prompt)
    torch.cuda.synchronize()
    ref = OB.block_decode(prompt, w, _odims(DIMS), cfg, draft, DIMS.mask_id)
    assert res.steps == ref["steps"] > 2
    assert res.accepted == ref["accepted"]
    assert res.unmasked == ref["unmasked"]
    np.testing.assert_array_equal(res.tokens, ref["tokens"])
    assert not (res.tokens == DIMS.mask_id).any()  # every block fully decoded
    np.testing.assert_array_equal(res.parent.tokens.cpu().numpy(), res.tokens)
    assert _rel(res.parent.layer_in.float().cpu().numpy(), ref["parent"]["layer_in"]) <= 2e-2
    got = res.parent.logits.float().cpu().numpy()
    assert _rel(got, ref["parent"]["logits"]) <= 2e-2 and _cos(got, ref["parent"]["logits"]) >= 0.999
    if acceptance_threshold > 0:
        assert min(res.stable_ratio) >= acceptance_threshold
