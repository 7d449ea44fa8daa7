"""Head-major parent keys and values (ParentCache.kv_hm, af_parent_kv_headmajor).

The parent cache keeps a second copy of each layer's K and V columns as
[2, n_kv_heads, T, 128], so the attention kernel reads a block of one head's
parent keys as one contiguous run. It is a layout of data the pass already
has, so:

* the copy equals the K / V columns of qkv exactly, after the parent pass and
  after a promotion rewrote rows of the cache;
* the folded pass gives bit-identical logits and stable masks (and scores
  equal up to the order of their fp32 atomic row sums) whether
  attention reads the head-major copy or the row-major qkv (LLaDA tiny,
  Dream tiny with GQA, and 2 layers of the LLaDA-8B shapes at 8 children x
  1024 tokens).
"""

from __future__ import annotations

import dataclasses

import pytest
import torch

from actfold_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _want_hm(pc, d):
    L, T = pc.qkv.shape[0], pc.seq
    k = pc.qkv[..., d.q_dim: d.q_dim + d.kv_dim].reshape(L, T, d.n_kv_heads, 128).permute(0, 2, 1, 3)
    v = pc.qkv[..., d.q_dim + d.kv_dim:].reshape(L, T, d.n_kv_heads, 128).permute(0, 2, 1, 3)
    return torch.stack([k, v], dim=1)


def _model_and_tokens(name):
    from actfold_b200.llada import LLaDAModel

    if name in ("llada-tiny", "dream-tiny"):
        dims = W.DIMS[name]
        parent, children = W.llada_tokens(64, 16, 0.5, 6, 4, dims.mask_id, 11)
        return LLaDAModel.from_numpy(dims, W.llada_weights_numpy(dims, seed=5), device="cuda", max_pos=64), parent, children
    dims = dataclasses.replace(W.LLADA_8B, n_layers=2)
    parent, _ = W.llada_tokens(1024, 256, 0.5, 1, 1, dims.mask_id, seed=42)
    children = W.llada_children(parent, 8, 16, dims.mask_id, seed=1000)
    return LLaDAModel.random(dims, seed=1234, device="cuda", max_pos=1024), parent, children


@pytest.mark.parametrize("name", ["llada-tiny", "dream-tiny", "llada8b_2layers"])
def test_folded_pass_is_the_same_with_either_layout(name):
    m, parent, children = _model_and_tokens(name)
    pc = m.parent_pass(torch.from_numpy(parent).cuda(), tau=0.95)
    assert torch.equal(pc.kv_hm, _want_hm(pc, m.dims))
    ct = torch.from_numpy(children).cuda()
    out = {}
    for hm in (True, False):
        m.kv_headmajor = hm
        m._plans = {}
        scores = torch.empty(ct.shape[0], dtype=torch.float32, device="cuda")
        logits, plan = m.verify(ct, pc, 0.95, scores=scores)
        assert bool(plan._pstruct.kv_headmajor) == hm
        torch.cuda.synchronize()
        plan.check_status()
        out[hm] = (logits.clone(), scores.clone(), plan.stable_masks().clone())
        del plan
    m.kv_headmajor = True
    m._plans = {}
    # Logits and masks bit for bit; scores are sums of fp32 row sums that the
    # LM-head epilogue adds with atomics, so only their last bits may differ.
    assert torch.equal(out[True][0], out[False][0])
    assert torch.equal(out[True][2], out[False][2])
    torch.testing.assert_close(out[True][1], out[False][1], rtol=1e-5, atol=0)


def test_promotion_keeps_the_copy_current():
    m, parent, children = _model_and_tokens("llada-tiny")
    pc = m.parent_pass(torch.from_numpy(parent).cuda(), tau=0.95)
    ct = torch.from_numpy(children).cuda()
    _, plan = m.verify(ct, pc, 0.95, keep_kv=True)
    pc2 = plan.promote(2)  # a copy: built from the clone's qkv, then the promoted rows
    plan.promote(3, into=pc)  # in place
    torch.cuda.synchronize()
    for c in (pc2, pc):
        assert c._kv_hm_at == c.version
        assert torch.equal(c.kv_hm, _want_hm(c, m.dims))
    assert not torch.equal(pc2.kv_hm, pc.kv_hm)
    # An in-place rewrite from elsewhere marks the copy stale; the next plan rebuilds it in the same buffer.
    buf = pc.kv_hm.data_ptr()
    pc.qkv.add_(1)
    pc.contents_changed()
    m._plans = {}
    _, plan = m.verify(ct, pc, 0.95)
    torch.cuda.synchronize()
    assert pc.kv_hm.data_ptr() == buf and torch.equal(pc.kv_hm, _want_hm(pc, m.dims))
