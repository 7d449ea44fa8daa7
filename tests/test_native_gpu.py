"""Native batched folded pass (LLaDA / Dream architectures) against the oracle and the golden vectors.

Tolerances (bf16 hidden states and logits): max relative error <= 2e-2 of the
tensor's scale, logit cosine >= 0.999, argmax agreement >= 99.9% over the rows
whose oracle argmax is defined (top-2 margin above two bf16 ulps of the row's
scale: random-init tiny models have exact bf16 ties, which any summation order
may break either way). Masks are compared bit-exactly except for rows the
oracle places on the gate boundary.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from actfold_b200 import workloads as W
from gen_inputs import TINY_DREAM, TINY_LLADA
from oracle import folding as OF
from oracle import llada as OL
from oracle.gate import decision_boundary
from oracle.numerics import from_bf16_bits

pytestmark = pytest.mark.gpu


def _odims(d):
    return OL.LLaDADims(d.n_layers, d.hidden, d.n_heads, d.n_kv_heads, d.head_dim, d.ffn, d.vocab, d.rms_eps, d.rope_theta)


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-6))


def _cos(a, b):
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float(a @ b / math.sqrt((a @ a) * (b @ b)))


def _argmax_agreement(got, ref):
    """Fraction of rows with equal argmax, over rows whose reference top-2 margin exceeds
    two bf16 ulps of the row's largest magnitude (ties and near-ties have no defined argmax)."""
    got = got.reshape(-1, got.shape[-1]).astype(np.float64)
    ref = ref.reshape(-1, ref.shape[-1]).astype(np.float64)
    top2 = np.sort(ref, axis=-1)[:, -2:]
    scale = np.abs(ref).max(-1)
    ulp = np.exp2(np.floor(np.log2(np.maximum(scale, 1e-30))) - 7)
    defined = (top2[:, 1] - top2[:, 0]) > 2 * ulp
    assert defined.mean() >= 0.75, "too few rows with a defined argmax to judge"
    return float((got.argmax(-1) == ref.argmax(-1))[defined].mean())


def _case(which):
    if which == "llada":
        return W.LLADA_TINY, TINY_LLADA, "llada_tiny"
    return W.DREAM_TINY, TINY_DREAM, "dream_tiny"


@pytest.fixture(scope="module", params=["llada", "dream"])
def tiny(request):
    from actfold_b200.llada import LLaDAModel

    dims, spec, gname = _case(request.param)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    parent, children = W.llada_tokens(spec["T"], spec["n_prompt"], spec["mask_frac"], spec["n_children"], spec["d"], dims.mask_id, spec["token_seed"])
    model = LLaDAModel.from_numpy(dims, w, device="cuda", max_pos=spec["T"])
    od = _odims(dims)
    ref_par = OF.llada_parent(parent, w, od)
    ref = OF.llada_folded_children(children, ref_par, w, od, spec["tau"])
    return dict(dims=dims, spec=spec, gname=gname, w=w, parent=parent, children=children, model=model, ref_par=ref_par, ref=ref)


def test_parent_pass_matches_oracle(tiny, attn_kernel):
    m = tiny["model"]
    pc = m.parent_pass(torch.from_numpy(tiny["parent"]).cuda(), tau=tiny["spec"]["tau"])
    torch.cuda.synchronize()
    assert _rel(pc.layer_in.float().cpu().numpy(), tiny["ref_par"]["layer_in"]) <= 2e-2
    d = tiny["dims"]
    k_ref = tiny["ref_par"]["k"]
    k_got = pc.qkv[:, :, d.q_dim: d.q_dim + d.kv_dim].float().cpu().numpy()
    assert _rel(k_got, k_ref) <= 2e-2
    lg = pc.logits.float().cpu().numpy()
    assert _rel(lg, tiny["ref_par"]["logits"]) <= 2e-2
    assert _cos(lg, tiny["ref_par"]["logits"]) >= 0.999
    assert pc.self_stable.bool().all()
    np.testing.assert_allclose(pc.row_sums.cpu().numpy(), lg.sum(-1), rtol=1e-3, atol=1e-2)


@pytest.fixture(params=["auto", "stream"])
def attn_kernel(request):
    """Each folded-pass parity case also runs with the streaming attention kernel
    (one CTA per query tile and head, online softmax) forced wherever it applies."""
    from actfold_b200 import _lib

    lib = _lib.load()
    kind = {"auto": 0, "stream": 1}[request.param]
    _lib.check(lib.af_set_attention_kernel(kind))
    yield request.param
    _lib.check(lib.af_set_attention_kernel(0))


def test_folded_children_match_oracle_and_reference(tiny, golden, attn_kernel):
    m = tiny["model"]
    spec = tiny["spec"]
    pc = m.parent_pass(torch.from_numpy(tiny["parent"]).cuda(), tau=spec["tau"])
    ct = torch.from_numpy(tiny["children"]).cuda()
    scores = torch.empty(ct.shape[0], device="cuda")
    logits, plan = m.verify(ct, pc, spec["tau"], scores=scores)
    torch.cuda.synchronize()
    plan.check_status()
    masks = plan.stable_masks().cpu().numpy()
    ref = tiny["ref"]
    np.testing.assert_array_equal(masks, ref["masks"])
    g = golden(tiny["gname"])
    np.testing.assert_array_equal(masks, g["masks"])  # the reference's own decisions
    got = logits.float().cpu().numpy()
    assert _rel(got, ref["logits"]) <= 2e-2
    assert _cos(got, ref["logits"]) >= 0.999
    assert _argmax_agreement(got, ref["logits"]) >= 0.999
    ref_g = from_bf16_bits(g["logits_bits"])
    assert _rel(got, ref_g) <= 2e-2 and _cos(got, ref_g) >= 0.999
    # per-layer child states through the merge/scatter materialisation
    for layer in range(tiny["dims"].n_layers + 1):
        st = plan.materialize(layer).float().cpu().numpy()
        assert _rel(st, ref["states"][layer]) <= 2e-2, layer
    np.testing.assert_allclose(scores.cpu().numpy(), got.reshape(got.shape[0], -1).mean(-1), rtol=1e-3, atol=1e-4)
    # divergent counts per layer and child agree with the masks
    np.testing.assert_array_equal(plan.div_count.cpu().numpy(), (~masks).sum(-1))


def test_unchanged_children_are_parent_copies(tiny):
    m = tiny["model"]
    pc = m.parent_pass(torch.from_numpy(tiny["parent"]).cuda(), tau=0.95)
    ct = torch.from_numpy(np.repeat(tiny["parent"][None], 3, axis=0)).cuda()
    logits, plan = m.verify(ct, pc, 0.95)
    torch.cuda.synchronize()
    plan.check_status()
    assert int(plan.n_fresh0.item()) == 0
    assert torch.equal(logits, pc.logits[None].expand_as(logits))
    assert plan.stable_masks().all()


def test_tau_one_parent_rows_fail_their_own_gate(tiny):
    """tau = 1.0: an identical row is stable only if its bf16 self-similarity rounds above 1.0.

    Rows the parent fails on itself become candidates of every child at that
    layer (the self-unstable path), so the pass still reproduces the reference.
    """
    m = tiny["model"]
    pc = m.parent_pass(torch.from_numpy(tiny["parent"]).cuda(), tau=1.0)
    assert not pc.self_stable.bool().all()  # the self-unstable path is exercised
    ct = torch.from_numpy(tiny["children"][:2]).cuda()
    logits, plan = m.verify(ct, pc, 1.0)
    torch.cuda.synchronize()
    plan.check_status()
    od = _odims(tiny["dims"])
    ref = OF.llada_folded_children(tiny["children"][:2], tiny["ref_par"], tiny["w"], od, 1.0)
    masks = plan.stable_masks().cpu().numpy()
    # Self-similarities of identical rows all sit within a few f32 ulps of the bf16
    # boundary 1.00390625, so accumulation order decides many of them; only the
    # bulk agreement and the outputs are meaningful here.
    assert (masks == ref["masks"]).mean() >= 0.95
    got = logits.float().cpu().numpy()
    assert _cos(got, ref["logits"]) >= 0.999
    assert (got.argmax(-1) == ref["logits"].argmax(-1)).mean() >= 0.97  # near-flat random-init logits


def test_self_unstable_rows_exact():
    """A zero embedding row makes the parent fail its own gate (sim 0) at layer 0: exact masks."""
    from actfold_b200.llada import LLaDAModel

    dims, spec = W.LLADA_TINY, TINY_LLADA
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    parent, children = W.llada_tokens(spec["T"], spec["n_prompt"], spec["mask_frac"], spec["n_children"], spec["d"], dims.mask_id, spec["token_seed"])
    w["embed"][parent[3]] = 0.0  # token at position 3 (and wherever else it occurs) has a zero embedding
    model = LLaDAModel.from_numpy(dims, w, device="cuda", max_pos=spec["T"])
    pc = model.parent_pass(torch.from_numpy(parent).cuda(), tau=spec["tau"])
    ss = pc.self_stable.cpu().numpy()
    assert not ss[0, 3]
    logits, plan = model.verify(torch.from_numpy(children).cuda(), pc, spec["tau"])
    torch.cuda.synchronize()
    plan.check_status()
    od = _odims(dims)
    ref = OF.llada_folded_children(children, OF.llada_parent(parent, w, od), w, od, spec["tau"])
    np.testing.assert_array_equal(plan.stable_masks().cpu().numpy(), ref["masks"])
    got = logits.float().cpu().numpy()
    assert _rel(got, ref["logits"]) <= 2e-2 and _cos(got, ref["logits"]) >= 0.999


def test_folded_model_api_on_llada(tiny):
    from actfold_b200.core import ActivationCache, FoldedModel, SimilarityGate
    from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER

    m = tiny["model"]
    cache = ActivationCache(max_entries_per_layer=1 << 20, device="cuda")
    fm = FoldedModel(m, cache, SimilarityGate(tau=0.95))
    assert fm.folding_applied
    GLOBAL_STABILITY_PROFILER.reset()
    pl = fm(torch.from_numpy(tiny["parent"])[None].cuda(), branch_id="parent")
    assert pl.shape == (1, tiny["spec"]["T"], tiny["dims"].vocab)
    # the parent's activations are visible through the cache API
    ones = torch.ones(1, tiny["spec"]["T"], dtype=torch.bool, device="cuda")
    got = cache.get("parent", 0, ones)
    assert set(got) == {"ffn_out", "hidden_states"}
    ids = [f"c{i}" for i in range(tiny["children"].shape[0])]
    lg = fm(torch.from_numpy(tiny["children"]).cuda(), branch_id=ids, parent_branch_id="parent")
    ref = tiny["ref"]
    assert _cos(lg.float().cpu().numpy(), ref["logits"]) >= 0.999
    prof = GLOBAL_STABILITY_PROFILER.get_profile("c0")
    assert len(prof.layer_stats) == tiny["dims"].n_layers
    assert prof.layer_stats[0].stable_ratio == pytest.approx(ref["masks"][0, 0].mean())


def test_gate_boundary_exemption_documented():
    # bf16 decision boundary at tau=0.95 is the midpoint between bf16(0.95) and the next bf16 value.
    assert decision_boundary(0.95, "bf16") == pytest.approx((0.94921875 + 0.953125) / 2)


def test_engine_graph_replay_matches_eager_launches(tiny):
    """verify_tokens replays a CUDA graph of the pass: for two different child batches in a row it
    must return exactly what the kernel-by-kernel launch returns (scores, divergent counts, logits)."""
    from actfold_b200.core import SimilarityGate
    from actfold_b200.speculative import ActFoldVerificationEngine, Branch

    model, spec, dims = tiny["model"], tiny["spec"], tiny["dims"]
    parent = torch.from_numpy(tiny["parent"])
    kids = tiny["children"]
    others = W.llada_children(tiny["parent"], kids.shape[0], spec["d"] + 1, dims.mask_id, seed=77)
    eng_g = ActFoldVerificationEngine(model, gate=SimilarityGate(spec["tau"]), use_graphs=True)
    eng_e = ActFoldVerificationEngine(model, gate=SimilarityGate(spec["tau"]), use_graphs=False)
    pb = Branch("parent", None, parent.reshape(1, -1))
    for batch in (kids, others, kids):
        host = torch.from_numpy(np.ascontiguousarray(batch)).pin_memory()
        rg = eng_g.verify_tokens(pb, host)
        rg_logits = rg["logits"].clone()
        re = eng_e.verify_tokens(pb, host)
        np.testing.assert_array_equal(rg["div_count"], re["div_count"])
        np.testing.assert_allclose(rg["scores"], re["scores"], rtol=1e-5, atol=1e-6)
        assert torch.equal(rg_logits.view(torch.int16), re["logits"].view(torch.int16))
