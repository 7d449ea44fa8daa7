"""Promotion of a verified child to a parent (chained folding) against the oracle and the reference.

The reference caches every verified child's merged per-layer activations under
the child's branch id (actfold/core/folded_transformer.py:190-199), so a later
verification may name the child as its parent. ``FoldPlan.promote`` builds
that parent cache on the device from the pass's fresh rows; these tests fold
grandchildren against it and compare with the oracle's chain and with the
reference's own chained run (tests/golden/llada_chain.npz).

Tolerances as in test_native_gpu: masks bit-exact except rows on the gate
boundary, bf16 logits max relative error <= 2e-2, cosine >= 0.999, argmax
agreement >= 99.9% over rows with a defined argmax.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from actfold_b200 import workloads as W
from gen_inputs import TINY_LLADA_CHAIN
from oracle import folding as OF
from oracle.numerics import from_bf16_bits
from test_native_gpu import _argmax_agreement, _cos, _odims, _rel

pytestmark = pytest.mark.gpu

SPEC = TINY_LLADA_CHAIN
DIMS = W.LLADA_TINY


@pytest.fixture(scope="module")
def chain():
    from actfold_b200.llada import LLaDAModel

    w = W.llada_weights_numpy(DIMS, seed=SPEC["weight_seed"])
    parent, children = W.llada_tokens(SPEC["T"], SPEC["n_prompt"], SPEC["mask_frac"], SPEC["n_children"], SPEC["d"],
                                      DIMS.mask_id, SPEC["token_seed"])
    k = SPEC["chain_child"]
    grand = W.llada_children(children[k], SPEC["chain_n"], SPEC["chain_d"], DIMS.mask_id, SPEC["chain_seed"])
    od = _odims(DIMS)
    ref = OF.llada_folded_children(children, OF.llada_parent(parent, w, od), w, od, SPEC["tau"])
    ref2 = OF.llada_folded_children(grand, OF.llada_promote(ref, k), w, od, SPEC["tau"])
    model = LLaDAModel.from_numpy(DIMS, w, device="cuda", max_pos=SPEC["T"])
    return dict(w=w, parent=parent, children=children, k=k, grand=grand, ref=ref, ref2=ref2, model=model)


def _check_grand(masks, logits, chain, golden):
    g = golden("llada_chain")
    np.testing.assert_array_equal(masks, chain["ref2"]["masks"])
    np.testing.assert_array_equal(masks, g["masks"])  # the reference's own chained decisions
    got = logits.float().cpu().numpy()
    for ref in (chain["ref2"]["logits"], from_bf16_bits(g["logits_bits"])):
        assert _rel(got, ref) <= 2e-2
        assert _cos(got, ref) >= 0.999
        assert _argmax_agreement(got, ref) >= 0.999


def test_promote_copy_then_fold_grandchildren(chain, golden):
    m = chain["model"]
    tau, k = SPEC["tau"], chain["k"]
    pc = m.parent_pass(torch.from_numpy(chain["parent"]).cuda(), tau=tau)
    before = [t.clone() for t in pc.tensors()]
    ct = torch.from_numpy(chain["children"]).cuda()
    logits, plan = m.verify(ct, pc, tau, keep_kv=True)
    pc2 = plan.promote(k)
    torch.cuda.synchronize()
    plan.check_status()
    # the source parent is untouched
    for a, b in zip(before, pc.tensors()):
        assert torch.equal(a, b)
    np.testing.assert_array_equal(pc2.tokens.cpu().numpy(), chain["children"][k])
    assert _rel(pc2.layer_in.float().cpu().numpy(), chain["ref"]["states"][:, k]) <= 2e-2
    # promoted logits are the child's own logits, bit for bit, with matching row sums
    assert torch.equal(pc2.logits, logits[k])
    np.testing.assert_allclose(pc2.row_sums.cpu().numpy(), pc2.logits.float().sum(-1).cpu().numpy(), rtol=1e-3, atol=1e-2)
    assert pc2.self_stable.bool().all()
    # QKV rows: unchanged rows keep the parent's; each fresh row is the QKV of the child's row
    d = DIMS
    fresh = (pc2.layer_in[:-1] != pc.layer_in[:-1]).any(-1)  # [L, T]
    assert fresh[0].cpu().numpy().tolist() == (chain["children"][k] != chain["parent"]).tolist()
    same = ~fresh
    assert torch.equal(pc2.qkv[same], pc.qkv[same])
    assert not torch.equal(pc2.qkv[fresh], pc.qkv[fresh])
    # grandchildren folded against the promoted child
    lg2, plan2 = m.verify(torch.from_numpy(chain["grand"]).cuda(), pc2, tau)
    torch.cuda.synchronize()
    plan2.check_status()
    _check_grand(plan2.stable_masks().cpu().numpy(), lg2, chain, golden)
    assert d.q_dim == pc2.qkv.shape[-1] - 2 * d.kv_dim


def test_promote_in_place_reuses_the_plan(chain, golden):
    m = chain["model"]
    tau, k = SPEC["tau"], chain["k"]
    pc = m.parent_pass(torch.from_numpy(chain["parent"]).cuda(), tau=tau)
    n = chain["children"].shape[0]
    ct = torch.from_numpy(chain["children"]).cuda()
    _, plan = m.verify(ct, pc, tau, keep_kv=True, m_cap=16)
    out = plan.promote(k, into=pc)
    assert out is pc
    # grandchildren (padded to the plan's child count with copies of the promoted child) on the same plan
    grand = np.repeat(chain["children"][k][None], n, axis=0)
    grand[: chain["grand"].shape[0]] = chain["grand"]
    lg2, plan2 = m.verify(torch.from_numpy(grand).cuda(), pc, tau, keep_kv=True, m_cap=16)
    assert plan2 is plan
    torch.cuda.synchronize()
    plan2.check_status()
    G = chain["grand"].shape[0]
    masks = plan2.stable_masks().cpu().numpy()
    assert masks[:, G:].all()  # unchanged copies of the new parent never diverge
    _check_grand(masks[:, :G], lg2[:G], chain, golden)
    assert torch.equal(lg2[G:], pc.logits[None].expand(n - G, -1, -1))


def test_engine_verifies_against_a_cache_promoted_in_place(chain, golden):
    """verify_tokens -> plan.promote(k, into=the engine's parent cache) -> verify_tokens on the promoted branch.

    The promotion rewrites the cache's token ids and self-gate rows on the
    device; the engine must see the new ids (not a stale host copy) when it
    matches the branch and sizes the next plan, and verify the grandchildren
    against the promoted child like the oracle's chain.
    """
    from actfold_b200.core import SimilarityGate
    from actfold_b200.speculative import ActFoldVerificationEngine, Branch

    m = chain["model"]
    tau, k = SPEC["tau"], chain["k"]
    eng = ActFoldVerificationEngine(m, gate=SimilarityGate(tau=tau), use_graphs=True)
    pb = Branch("p", None, torch.from_numpy(chain["parent"])[None])
    kids = torch.from_numpy(chain["children"]).pin_memory()
    res = eng.verify_tokens(pb, kids)
    res["plan"].keep_kv()
    res = eng.verify_tokens(pb, kids)  # recaptured: this run keeps its QKV rows
    pc = eng.parent_cache(pb)
    res["plan"].promote(k, into=pc)
    kb = Branch("p", None, torch.from_numpy(chain["children"][k])[None])
    assert eng.parent_cache(kb) is pc  # matched on the promoted ids, no new dense pass
    res2 = eng.verify_tokens(kb, torch.from_numpy(chain["grand"]).pin_memory())
    torch.cuda.synchronize()
    _check_grand(res2["plan"].stable_masks().cpu().numpy(), res2["logits"], chain, golden)


def test_folded_model_chains_through_a_verified_child(chain, golden):
    from actfold_b200.core import ActivationCache, FoldedModel, SimilarityGate

    m = chain["model"]
    k = chain["k"]
    cache = ActivationCache(max_entries_per_layer=1 << 16, device="cuda")
    fm = FoldedModel(m, cache, SimilarityGate(tau=SPEC["tau"]))
    fm(torch.from_numpy(chain["parent"])[None].cuda(), branch_id="parent")
    ids = [f"child{i}" for i in range(chain["children"].shape[0])]
    fm(torch.from_numpy(chain["children"]).cuda(), branch_id=ids, parent_branch_id="parent")
    gids = [f"grand{i}" for i in range(chain["grand"].shape[0])]
    lg = fm(torch.from_numpy(chain["grand"]).cuda(), branch_id=gids, parent_branch_id=f"child{k}")
    from actfold_b200.profiler import GLOBAL_STABILITY_PROFILER

    g = golden("llada_chain")
    for i, gid in enumerate(gids):
        prof = GLOBAL_STABILITY_PROFILER.get_profile(gid)
        assert prof is not None and prof.parent_branch_id == f"child{k}"
        ratios = [s.stable_ratio for s in prof.layer_stats]
        np.testing.assert_allclose(ratios, g["masks"][:, i].mean(-1), atol=1e-6)
    got = lg.float().cpu().numpy()
    ref = from_bf16_bits(g["logits_bits"])
    assert _rel(got, ref) <= 2e-2 and _cos(got, ref) >= 0.999 and _argmax_agreement(got, ref) >= 0.999
    # the promoted child is visible through the cache API, like the reference's stored child entries
    ones = torch.ones(1, SPEC["T"], dtype=torch.bool, device="cuda")
    assert set(cache.get(f"child{k}", 0, ones)) == {"ffn_out", "hidden_states"}
    cache.clear_branch(f"child{k}")
    assert f"child{k}" not in cache.native_parents and f"child{k}" not in cache.native_children


@pytest.mark.parametrize("name", ["longer", "shorter"])
def test_children_of_another_length_fold_like_the_reference(golden, name):
    """A child longer than its parent folds against zero-filled parent rows; a shorter one against a prefix."""
    from actfold_b200.core import ActivationCache, FoldedModel, SimilarityGate
    from actfold_b200.llada import LLaDAModel
    from gen_inputs import TINY_LLADA_RESIZE

    g = golden("llada_resize")
    spec = TINY_LLADA_RESIZE
    w = W.llada_weights_numpy(DIMS, seed=spec["weight_seed"])
    model = LLaDAModel.from_numpy(DIMS, w, device="cuda", max_pos=64)
    fm = FoldedModel(model, ActivationCache(max_entries_per_layer=1 << 16, device="cuda"), SimilarityGate(tau=spec["tau"]))
    fm(torch.from_numpy(g["parent"])[None].cuda(), branch_id="parent")
    kids = g[name]
    lg = fm(torch.from_numpy(kids).cuda(), branch_id=[f"{name}{i}" for i in range(kids.shape[0])], parent_branch_id="parent")
    torch.cuda.synchronize()
    od = _odims(DIMS)
    ref = OF.llada_folded_children(kids, OF.llada_resize_parent(OF.llada_parent(g["parent"], w, od), kids.shape[1]), w, od,
                                   spec["tau"])
    np.testing.assert_array_equal(ref["masks"], g[f"{name}_masks"])
    got = lg.float().cpu().numpy()
    for want in (ref["logits"], from_bf16_bits(g[f"{name}_logits_bits"])):
        assert _rel(got, want) <= 2e-2 and _cos(got, want) >= 0.999 and _argmax_agreement(got, want) >= 0.999
    from actfold_b200.profiler import GLOBAL_STABILITY_PROFILER

    for i in range(kids.shape[0]):
        prof = GLOBAL_STABILITY_PROFILER.get_profile(f"{name}{i}")
        np.testing.assert_allclose([s.stable_ratio for s in prof.layer_stats], g[f"{name}_masks"][:, i].mean(-1), atol=1e-6)


def test_autoregressive_chain_folds_natively(chain):
    """Greedy next-token generation as folded_generate runs it (speculative/folded_generation.py:44-138):
    each step's child is the previous branch plus one token, verified with the previous branch as its parent.

    Every step folds on the native pass (a one-row-longer child against the zero-filled, promoted parent)
    and matches the oracle chain (resize + fold + promote) on the same tokens.
    """
    from actfold_b200.core import ActivationCache, FoldedModel, SimilarityGate

    m, w = chain["model"], chain["w"]
    od = _odims(DIMS)
    cache = ActivationCache(max_entries_per_layer=1 << 16, device="cuda")
    fm = FoldedModel(m, cache, SimilarityGate(tau=SPEC["tau"]))
    tokens = chain["parent"][:56].copy()
    logits = fm(torch.from_numpy(tokens)[None].cuda(), branch_id="root")
    ref_parent = OF.llada_parent(tokens, w, od)
    pid = "root"
    for step in range(4):
        nxt = int(logits[0, -1].float().argmax())
        tokens = np.concatenate([tokens, [nxt]])
        cid = f"{pid}/t{step}/d0"
        logits = fm(torch.from_numpy(tokens)[None].cuda(), branch_id=cid, parent_branch_id=pid)
        assert cid in cache.native_children  # verified on the folded pass, promotable
        ref = OF.llada_folded_children(tokens[None], OF.llada_resize_parent(ref_parent, tokens.size), w, od, SPEC["tau"])
        assert (~ref["masks"][0, 0]).sum() == 1 and not ref["masks"][0, 0, -1]  # only the new token diverges at layer 0
        got = logits[0].float().cpu().numpy()
        assert _rel(got, ref["logits"][0]) <= 2e-2 and _cos(got, ref["logits"][0]) >= 0.999
        ref_parent = OF.llada_promote(ref, 0)
        pid = cid
