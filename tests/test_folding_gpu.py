"""Generic folded path on the GPU: the reference's layer / wrapper tests and the demo workload.

Layer tests follow tests/test_folded_transformer.py:29-132 and
tests/test_model_wrapper.py of the reference, run on CUDA tensors. The demo
test runs FoldedModel over the demo.py model (fp32) and compares per-layer
masks and logits with the golden vectors recorded from the reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn

from actfold_b200 import workloads as W
from demo_model import SyntheticTransformer, load_demo_weights
from gen_inputs import DEMO

pytestmark = pytest.mark.gpu


class DummyLayer(nn.Module):
    def __init__(self, hidden_dim: int) -> None:
        super().__init__()
        self.linear = nn.Linear(hidden_dim, hidden_dim, bias=False)
        with torch.no_grad():
            self.linear.weight.copy_(torch.eye(hidden_dim))

    def forward(self, hidden_states, attention_mask=None):
        return self.linear(hidden_states)


class TupleOutputLayer(nn.Module):
    def forward(self, hidden_states, attention_mask=None):
        return hidden_states * 2, hidden_states


def _mk(layer, tau=0.95, scheduler=None):
    from actfold_b200.core import ActivationCache, FoldedTransformerLayer, SimilarityGate

    cache = ActivationCache(device="cuda")
    return FoldedTransformerLayer(layer.cuda(), cache, SimilarityGate(tau=tau), layer_idx=0, scheduler=scheduler), cache


def test_layer_without_parent():
    folded, _ = _mk(DummyLayer(32))
    x = torch.randn(2, 8, 32, device="cuda")
    torch.testing.assert_close(folded(x, branch_id="root"), folded.original_layer(x), atol=1e-5, rtol=0)


def test_layer_tuple_output():
    folded, _ = _mk(TupleOutputLayer())
    x = torch.randn(2, 4, 16, device="cuda")
    torch.testing.assert_close(folded(x, branch_id="root"), x * 2)


def test_layer_with_parent_near_identical_child():
    folded, cache = _mk(DummyLayer(32))
    parent = torch.randn(2, 8, 32, device="cuda")
    parent_out = folded(parent, branch_id="parent")
    cache.put("parent", 0, {"ffn_out": parent_out, "hidden_states": parent})
    child = parent + 1e-5 * torch.randn_like(parent)
    out = folded(child, branch_id="child", parent_branch_id="parent")
    assert out.shape == (2, 8, 32)
    torch.testing.assert_close(out, parent_out, atol=1e-3, rtol=0)


def test_layer_divergent_only():
    folded, _ = _mk(DummyLayer(16), tau=0.99)
    parent = torch.randn(2, 4, 16, device="cuda")
    folded(parent, branch_id="parent")
    child = torch.randn(2, 4, 16, device="cuda")
    torch.testing.assert_close(folded(child, branch_id="child", parent_branch_id="parent"), folded.original_layer(child), atol=1e-5, rtol=0)


def test_layer_partial_merge_matches_where():
    folded, _ = _mk(DummyLayer(64).to(torch.bfloat16))
    parent = torch.randn(3, 16, 64, device="cuda").to(torch.bfloat16)
    pout = folded(parent, branch_id="parent")
    child = parent.clone()
    child[:, 5] = torch.randn(3, 64, device="cuda").to(torch.bfloat16)
    out = folded(child, branch_id="child", parent_branch_id="parent")
    from actfold_b200.core import SimilarityGate

    m = SimilarityGate(0.95)(child, parent)
    assert (~m).sum() >= 3
    torch.testing.assert_close(out, torch.where(m[..., None], pout, folded.original_layer(child)), rtol=0, atol=0)


def test_layer_scheduler_disables_layer():
    from actfold_b200.core import FoldingScheduler

    sch = FoldingScheduler(base_tau=0.95, num_layers=2, num_steps=1)
    sch.disable_layers([0])
    folded, _ = _mk(DummyLayer(16), scheduler=sch)
    parent = torch.randn(2, 4, 16, device="cuda")
    folded(parent, branch_id="parent")
    child = parent.clone()
    torch.testing.assert_close(folded(child, branch_id="child", parent_branch_id="parent", step_idx=0), folded.original_layer(child), atol=1e-5, rtol=0)


def test_layer_with_chunked_cache_partial_mask():
    """The reference raises 'Shape mismatch' here; the chunked cache folds correctly in this build."""
    from actfold_b200.core import ChunkedActivationCache, FoldedTransformerLayer, SimilarityGate

    cache = ChunkedActivationCache(max_entries_per_layer=4096, chunk_size=64, device="cuda")
    folded = FoldedTransformerLayer(DummyLayer(64).cuda(), cache, SimilarityGate(0.95), 0)
    parent = torch.randn(1, 128, 64, device="cuda")
    pout = folded(parent, branch_id="p")
    child = parent.clone()
    child[:, 4] = torch.randn(64, device="cuda")
    out = folded(child, branch_id="c", parent_branch_id="p")
    torch.testing.assert_close(out[:, 4], folded.original_layer(child)[:, 4], atol=1e-5, rtol=0)
    torch.testing.assert_close(out[:, 5:], pout[:, 5:], rtol=0, atol=0)


def _demo_models():
    from actfold_b200.core import ActivationCache, FoldedModel, SimilarityGate

    w = W.demo_weights(seed=DEMO["weight_seed"])
    base = load_demo_weights(SyntheticTransformer(), w).cuda().eval()
    cache = ActivationCache(max_entries_per_layer=1024, device="cuda")
    folded = FoldedModel(load_demo_weights(SyntheticTransformer(), w).cuda().eval(), cache, SimilarityGate(tau=DEMO["tau"]))
    return base, folded


def test_demo_workload_matches_reference_golden(golden):
    from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER

    g = golden("demo")
    base, folded = _demo_models()
    assert folded.folding_applied
    parent, children = W.demo_tokens(seed=DEMO["token_seed"], T=DEMO["T"], n_children=DEMO["n_children"])
    GLOBAL_STABILITY_PROFILER.reset()
    with torch.no_grad():
        pl = folded(torch.from_numpy(parent)[None].cuda(), branch_id="parent")
        np.testing.assert_allclose(pl[0].cpu().numpy(), g["parent_logits"], rtol=2e-3, atol=2e-4)
        for c in range(children.shape[0]):
            ct = torch.from_numpy(children[c])[None].cuda()
            lg = folded(ct, branch_id=f"child{c}", parent_branch_id="parent")
            np.testing.assert_allclose(lg[0].cpu().numpy(), g["logits"][c], rtol=2e-3, atol=2e-4)
            prof = GLOBAL_STABILITY_PROFILER.get_profile(f"child{c}")
            m = np.ones((4, DEMO["T"]), bool)
            for st in prof.layer_stats:
                if st.divergence_positions is not None:
                    for _, t in st.divergence_positions.tolist():
                        m[st.layer_idx, t] = False
            np.testing.assert_array_equal(m, g["masks"][:, c])
            bl = base(ct)
            mse = float((bl - lg).pow(2).mean())
            assert mse < 1e-2


def test_wrapper_restore_and_passthrough():
    from actfold_b200.core import ActivationCache, FoldedModel, SimilarityGate

    base = SyntheticTransformer().cuda()
    fm = FoldedModel(base, ActivationCache(device="cuda"), SimilarityGate())
    from actfold_b200.core import FoldedTransformerLayer

    assert isinstance(base.layers[0], FoldedTransformerLayer)
    restored = fm.restore()
    assert not isinstance(restored.layers[0], FoldedTransformerLayer)

    class NoLayers(nn.Module):
        def forward(self, tokens):
            return tokens.float() * 2

    with pytest.warns(UserWarning):
        fm2 = FoldedModel(NoLayers(), ActivationCache(device="cuda"), SimilarityGate())
    assert not fm2.folding_applied
    t = torch.ones(1, 3, dtype=torch.long, device="cuda")
    torch.testing.assert_close(fm2(t, branch_id="x"), t.float() * 2)
