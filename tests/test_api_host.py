"""Host-side behaviour of the drop-in API (CPU only: validation, errors, bookkeeping).

Mirrors the error conventions pinned by the reference's tests
(tests/test_similarity_gate.py:52-77, test_fused_ops.py:63-77,
test_activation_cache.py:70-86, test_chunked_cache.py:62-68,
test_folding_scheduler.py, test_stability_profiler.py). Any call that would
compute requires CUDA tensors and must say so instead of falling back.
"""

from __future__ import annotations

import pytest
import torch

from actfold_b200.core import (
    ActivationCache,
    ChunkedActivationCache,
    FoldedTransformerLayer,
    FoldingScheduler,
    SimilarityGate,
    make_activation_cache,
    merge_stable_divergent,
)
from actfold_b200.core.folding_context import FOLDING_CONTEXT, folding_scope
from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER, StabilityProfiler


def test_gate_constructor_errors():
    with pytest.raises(ValueError, match="tau must be in"):
        SimilarityGate(tau=1.5)
    with pytest.raises(ValueError, match="Unsupported metric"):
        SimilarityGate(metric="manhattan")


def test_gate_shape_errors_before_device_checks():
    g = SimilarityGate()
    with pytest.raises(ValueError, match="Shape mismatch"):
        g(torch.randn(1, 4, 8), torch.randn(1, 4, 16))
    with pytest.raises(ValueError, match="3-D"):
        g(torch.randn(4, 8), torch.randn(4, 8))


def test_gate_set_tau():
    g = SimilarityGate(tau=0.9)
    g.set_tau(0.5)
    assert g.tau == 0.5
    with pytest.raises(ValueError):
        g.set_tau(-0.1)
    assert "tau=0.5" in g.extra_repr()


def test_gate_refuses_cpu_tensors():
    with pytest.raises(RuntimeError, match="CUDA"):
        SimilarityGate()(torch.randn(1, 4, 8), torch.randn(1, 4, 8))


def test_merge_shape_errors():
    p = torch.randn(2, 8, 32)
    with pytest.raises(ValueError):
        merge_stable_divergent(p, torch.randn(2, 8, 64), torch.ones(2, 8, dtype=torch.bool))
    with pytest.raises(ValueError):
        merge_stable_divergent(p, torch.randn(2, 4, 32), torch.ones(2, 8, dtype=torch.bool))
    with pytest.raises(ValueError):
        merge_stable_divergent(p, torch.randn(2, 8, 32), torch.ones(2, 4, dtype=torch.bool))
    with pytest.raises(RuntimeError, match="CUDA"):
        merge_stable_divergent(p, torch.randn(2, 8, 32), torch.ones(2, 8, dtype=torch.bool))


def test_cache_put_validation():
    cache = ActivationCache(device="cpu")
    with pytest.raises(ValueError, match="activations must not be empty"):
        cache.put("a", 0, {})
    with pytest.raises(ValueError, match="inconsistent leading shape"):
        cache.put("a", 0, {"ffn_out": torch.randn(1, 4, 8), "hidden_states": torch.randn(1, 3, 8)})
    with pytest.raises(ValueError, match="at least 2 leading"):
        cache.put("a", 0, {"ffn_out": torch.randn(4)})
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.put("a", 0, {"ffn_out": torch.randn(1, 4, 8)})


def test_cache_missing_branch_raises_keyerror():
    cache = ActivationCache(device="cpu")
    with pytest.raises(KeyError):
        cache.get("missing", 0, torch.ones(1, 2, dtype=torch.bool))
    assert cache.num_entries() == 0


def test_chunked_cache_validation_and_empty_get():
    with pytest.raises(ValueError):
        ChunkedActivationCache(chunk_size=0)
    with pytest.raises(ValueError):
        ChunkedActivationCache(max_entries_per_layer=0)
    c = ChunkedActivationCache(max_entries_per_layer=128, chunk_size=4, device="cpu")
    assert c.get("b", 0, torch.ones(1, 4, dtype=torch.bool)) == {}
    assert c.num_tokens() == 0


def test_cache_factory():
    assert isinstance(make_activation_cache(16, "cpu"), ActivationCache)
    c = make_activation_cache(16, "cpu", use_chunked=True, chunk_size=4)
    assert isinstance(c, ChunkedActivationCache) and c.max_chunks == 4


def test_scheduler_matches_reference_schedule():
    s = FoldingScheduler(base_tau=0.95, num_layers=12, num_steps=10)
    assert s.get_tau(0, 9) == pytest.approx(min(max(0.95 + 0.03, 0.80), 0.99))
    assert s.get_tau(11, 0) == pytest.approx(0.95 - 0.03 - 0.04)
    assert not s.should_fold(11, 0) and not s.should_fold(0, 9) and s.should_fold(0, 0)
    s.disable_layers({3})
    assert not s.should_fold(3, 0)
    s.enable_layers({3})
    assert s.should_fold(3, 0)
    with pytest.raises(ValueError):
        s.get_tau(12, 0)
    with pytest.raises(ValueError):
        FoldingScheduler(base_tau=2.0)


def test_profiler_records_and_flushes_lazily():
    prof = StabilityProfiler(enabled=True)
    prof.record("child", "parent", layer_idx=1, step_idx=0, stable_mask=torch.tensor([[True, True, False, True]]), tau=0.95)
    assert len(prof._pending) == 1
    p = prof.get_profile("child")
    assert p.layer_stats[0].stable_ratio == pytest.approx(0.75)
    assert p.layer_stats[0].divergence_positions.tolist() == [[0, 2]]
    assert p.mean_stable_ratio == pytest.approx(0.75)
    prof.record("b2", None, 1, 0, torch.zeros(1, 2, dtype=torch.bool), 0.9)
    assert prof.get_mean_stable_ratio(1, 0) == pytest.approx(0.375)
    assert prof.get_mean_stable_ratio(5, 0) is None


def test_profiler_record_batch():
    prof = StabilityProfiler()
    masks = torch.ones(3, 2, 4, dtype=torch.bool)
    masks[1, 0, 2] = False
    prof.record_batch(["c0", "c1"], "p", 0, masks, 0.95)
    p0 = prof.get_profile("c0")
    assert [s.layer_idx for s in p0.layer_stats] == [0, 1, 2]
    assert p0.layer_stats[1].stable_ratio == pytest.approx(0.75)
    assert prof.get_profile("c1").min_stable_ratio == 1.0


def test_profiler_disabled_and_global_reset():
    prof = StabilityProfiler(enabled=False)
    prof.record("c", "p", 0, 0, torch.ones(1, 4, dtype=torch.bool), 0.95)
    assert prof.get_profile("c") is None
    GLOBAL_STABILITY_PROFILER.record("c", "p", 0, 0, torch.ones(1, 2, dtype=torch.bool), 0.9)
    assert GLOBAL_STABILITY_PROFILER.get_profile("c") is not None
    GLOBAL_STABILITY_PROFILER.reset()
    assert GLOBAL_STABILITY_PROFILER.get_profile("c") is None


def test_folding_scope_sets_and_resets_context():
    assert FOLDING_CONTEXT.get() is None
    with folding_scope("c", "p", 3):
        assert FOLDING_CONTEXT.get() == {"branch_id": "c", "parent_branch_id": "p", "step_idx": 3}
    assert FOLDING_CONTEXT.get() is None


def test_folded_layer_requires_branch_id():
    layer = FoldedTransformerLayer(torch.nn.Identity(), ActivationCache(device="cpu"), SimilarityGate(), 0)
    with pytest.raises(ValueError, match="branch_id"):
        layer(torch.randn(1, 2, 4))
