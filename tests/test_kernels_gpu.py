"""GPU parity of the gate / compaction / row kernels against the oracle and the golden vectors."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from gen_inputs import GATE_CASES, digest, gate_inputs
from oracle.gate import compact, exempt_rows, gate
from oracle.numerics import from_bf16_bits
from oracle.rows import gather_dense, merge

pytestmark = pytest.mark.gpu

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _dev(a: np.ndarray, dt: str) -> torch.Tensor:
    return torch.from_numpy(a).to(TORCH_DT[dt]).cuda()


@pytest.mark.parametrize("case", GATE_CASES, ids=[c[0] for c in GATE_CASES])
def test_gate_kernel_matches_oracle_and_reference(golden, case):
    from actfold_b200.core import SimilarityGate

    name, seed, B, T, H, dt, tau, metric = case
    g = golden("gate")
    c, p = gate_inputs(seed, B, T, H, dt)
    assert str(g[f"{name}/digest"]) == digest(c, p)
    ora = gate(c, p, tau, metric, 1e-8, dt)
    sg = SimilarityGate(tau=tau, metric=metric)
    res = sg.forward_compact(_dev(c, dt), _dev(p, dt), stable_idx=True)
    mask = res.stable_mask.cpu().numpy()
    sim = sg.similarity(_dev(c, dt), _dev(p, dt)).cpu().numpy()
    # masks: bit-exact against the reference's own output except boundary rows
    ref_mask = g[f"{name}/mask"]
    ex = exempt_rows(ora)
    assert not ((mask != ref_mask) & ~ex).any(), f"{int((mask != ref_mask).sum())} mismatches vs reference"
    assert not ((mask != ora.mask) & ~ex).any()
    both_nan = np.isnan(sim) & np.isnan(ora.sim)
    if dt == "f32":
        # f32 sums differ from the oracle's only in accumulation order
        assert (np.isclose(sim, ora.sim, rtol=0, atol=2e-6) | both_nan).all()
    elif metric == "cosine":
        same = (sim == ora.sim) | both_nan
        assert same.mean() >= 0.999, same.mean()
    # compaction: order-preserving lists and counts equal the oracle's for this mask
    st, dv, cnt = compact(mask)
    np.testing.assert_array_equal(res.div_count.cpu().numpy(), cnt)
    di = res.div_idx.cpu().numpy()
    si = res.stable_idx.cpu().numpy()
    for b in range(B):
        np.testing.assert_array_equal(di[b, : cnt[b]], dv[b])
        assert (di[b, cnt[b]:] == -1).all()
        np.testing.assert_array_equal(si[b, : T - cnt[b]], st[b])
        assert (si[b, T - cnt[b]:] == -1).all()


def test_gate_bf16_edges_on_device():
    from actfold_b200.core import SimilarityGate

    x = torch.ones(1, 3, 64, dtype=torch.bfloat16, device="cuda")
    assert SimilarityGate(0.98)(x, x).all()
    assert not SimilarityGate(1.0)(x, x).any()
    # broadcast parent (stride 0 over the batch)
    p = torch.randn(1, 5, 256, device="cuda").to(torch.bfloat16)
    c = p.expand(4, 5, 256)
    assert SimilarityGate(0.95)(c, p.expand(4, 5, 256)).all()


@pytest.mark.parametrize("B,H", [(20, 4096), (3, 3584), (9, 1024)])
def test_gate_broadcast_parent_kernel(B, H):
    """A parent row shared by every child (batch stride 0) takes the broadcast kernel: the same similarity
    bits as the per-row kernel on a materialised parent, and the oracle's decisions."""
    from actfold_b200.core import SimilarityGate

    c, p = gate_inputs(40 + B, B, 64, H, "bf16")
    p1 = p[:1]
    sg = SimilarityGate(tau=0.95)
    tp = _dev(p1, "bf16")
    sim_b = sg.similarity(_dev(c, "bf16"), tp.expand(B, 64, H)).cpu().numpy()
    sim_r = sg.similarity(_dev(c, "bf16"), tp.expand(B, 64, H).contiguous()).cpu().numpy()
    np.testing.assert_array_equal(sim_b.view(np.uint32), sim_r.view(np.uint32))
    mask = sg(_dev(c, "bf16"), tp.expand(B, 64, H)).cpu().numpy()
    ora = gate(c, np.broadcast_to(p1, c.shape), 0.95, "cosine", 1e-8, "bf16")
    assert not ((mask != ora.mask) & ~exempt_rows(ora)).any()
    assert ((sim_b == ora.sim) | (np.isnan(sim_b) & np.isnan(ora.sim))).mean() >= 0.999


def test_gate_broadcast_extreme_magnitudes_match_oracle():
    """The broadcast kernel's packed chain (x * approximate 1/n, one bf16 rounding per product) against the
    oracle's exact chain on rows built to reach its edges: bf16 subnormal elements beside normal ones (their
    quotients are fp32 subnormals), a row of subnormals only (norm clamped to eps), zero elements and rows,
    rows whose squares overflow fp32 (norm inf), and a NaN element. Masks and similarity bits equal the
    oracle's on every row."""
    from actfold_b200.core import SimilarityGate
    from oracle.numerics import round_bf16

    B, T, H = 8, 16, 4096
    rng = np.random.default_rng(7)
    parent = rng.standard_normal((1, T, H), dtype=np.float32)
    child = np.repeat(parent, B, axis=0) + np.float32(0.05) * rng.standard_normal((B, T, H), dtype=np.float32)
    sub = np.float32(2.0 ** -133)  # smallest bf16 subnormal
    child[0, 0, ::7] = sub
    child[0, 1, ::3] = -sub
    child[1, 2] = sub * rng.integers(1, 100, H).astype(np.float32)  # subnormals only
    child[2, 3] = 0.0
    child[2, 4, ::2] = 0.0
    child[3, 5] *= np.float32(2.0 ** 70)  # squares overflow fp32
    child[4, 6, 100] = np.nan
    parent[0, 7, ::5] = sub  # the parent row itself holds subnormals
    child = round_bf16(child)
    parent = round_bf16(parent)
    sg = SimilarityGate(tau=0.95)
    tp = torch.from_numpy(parent).to(torch.bfloat16).cuda().expand(B, T, H)  # batch stride 0: broadcast kernel
    tc = torch.from_numpy(child).to(torch.bfloat16).cuda()
    sim = sg.similarity(tc, tp).cpu().numpy()
    mask = sg(tc, tp).cpu().numpy()
    ora = gate(child, np.broadcast_to(parent, child.shape), 0.95, "cosine", 1e-8, "bf16")
    same = (sim.view(np.uint32) == ora.sim.view(np.uint32)) | (np.isnan(sim) & np.isnan(ora.sim))
    edges = [(0, 0), (0, 1), (1, 2), (2, 3), (2, 4), (3, 5), (4, 6)] + [(b, 7) for b in range(B)]
    assert all(same[e] for e in edges), [e for e in edges if not same[e]]
    # Ordinary rows: the fp32 sums run in another order than the oracle's, which can move a similarity
    # across a bf16 rounding boundary only rarely.
    assert same.mean() >= 0.99, same.mean()
    assert not ((mask != ora.mask) & ~exempt_rows(ora)).any()


@pytest.mark.parametrize("H", [4096, 3584, 100])
def test_gate_large_and_odd_hidden(H):
    from actfold_b200.core import SimilarityGate

    c, p = gate_inputs(99, 2, 64, H, "bf16")
    ora = gate(c, p, 0.95, "cosine", 1e-8, "bf16")
    m = SimilarityGate(0.95)(_dev(c, "bf16"), _dev(p, "bf16")).cpu().numpy()
    assert not ((m != ora.mask) & ~exempt_rows(ora)).any()


def test_gate_empty_batch():
    from actfold_b200.core import SimilarityGate

    z = torch.empty(0, 4, 64, device="cuda", dtype=torch.bfloat16)
    assert SimilarityGate()(z, z).shape == (0, 4)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_merge_kernel_matches_reference(golden, dt):
    from actfold_b200.core import merge_stable_divergent

    g = golden("merge")
    out = merge_stable_divergent(_dev(g[f"{dt}/parent"], dt), _dev(g[f"{dt}/child"], dt), torch.from_numpy(g[f"{dt}/mask"]).cuda())
    np.testing.assert_array_equal(out.float().cpu().numpy(), g[f"{dt}/out"])


def test_merge_large_rows_and_broadcast_parent():
    from actfold_b200.core import merge_stable_divergent

    rng = np.random.default_rng(3)
    p = rng.standard_normal((1, 300, 4096), dtype=np.float32)
    c = rng.standard_normal((3, 300, 4096), dtype=np.float32)
    m = rng.random((3, 300)) > 0.3
    pt = _dev(p, "bf16").expand(3, 300, 4096)
    out = merge_stable_divergent(pt, _dev(c, "bf16"), torch.from_numpy(m).cuda())
    ref = merge(np.broadcast_to(_dev(p, "bf16").float().cpu().numpy(), c.shape), _dev(c, "bf16").float().cpu().numpy(), m)
    np.testing.assert_array_equal(out.float().cpu().numpy(), ref)


def test_merge_unaligned_rows_use_byte_path():
    from actfold_b200.core import merge_stable_divergent

    p = torch.randn(2, 7, 3, device="cuda")
    c = torch.randn(2, 7, 3, device="cuda")
    m = torch.rand(2, 7, device="cuda") > 0.5
    torch.testing.assert_close(merge_stable_divergent(p, c, m), torch.where(m[..., None], p, c), rtol=0, atol=0)


def test_cache_replays_reference_log(golden):
    from actfold_b200.core import ActivationCache

    g = golden("cache")
    log = json.loads(str(g["log"]))
    cache = ActivationCache(max_entries_per_layer=14, device="cuda")
    for rec in log:
        i = rec["i"]
        if rec["kind"] == "put":
            cache.put(rec["branch"], rec["layer"], {n: torch.from_numpy(g[f"{i}/in/{n}"]).cuda() for n in rec["names"]}, rec["step"])
        elif rec["kind"] == "get":
            m = torch.from_numpy(g[f"{i}/mask"]).cuda()
            if rec.get("keyerror"):
                with pytest.raises(KeyError):
                    cache.get(rec["branch"], rec["layer"], m, rec["step"])
            else:
                out = cache.get(rec["branch"], rec["layer"], m, rec["step"])
                assert sorted(out) == rec["out_names"]
                for n in rec["out_names"]:
                    np.testing.assert_array_equal(out[n].cpu().numpy(), g[f"{i}/out/{n}"])
        elif rec["kind"] == "clear_branch":
            cache.clear_branch(rec["branch"])
        elif rec["kind"] == "clear_layer":
            cache.clear_layer(rec["layer"])
        assert cache.num_entries() == rec["num_entries"], i
        assert cache.num_entries(0) == rec["num_entries_l0"], i


def test_gather_cached_activations_raw_dict_paths():
    from actfold_b200.core import gather_cached_activations

    cache = {("b", 0, t, 0): {"ffn_out": torch.randn(2, 32, device="cuda"), "hidden_states": torch.randn(2, 32, device="cuda")} for t in range(4)}
    mask = torch.tensor([[True, True, False, False], [False, True, True, True]], device="cuda")
    out = gather_cached_activations(cache, "b", 0, mask)
    stacked = np.stack([cache[("b", 0, t, 0)]["ffn_out"].cpu().numpy() for t in range(4)], axis=1)
    np.testing.assert_array_equal(out["ffn_out"].cpu().numpy(), gather_dense(stacked, mask.cpu().numpy()))
    del cache[("b", 0, 2, 0)]
    out = gather_cached_activations(cache, "b", 0, torch.ones(2, 4, dtype=torch.bool, device="cuda"))
    assert (out["ffn_out"][:, 2] == 0).all()
    with pytest.raises(KeyError):
        gather_cached_activations({}, "b", 0, torch.ones(1, 4, dtype=torch.bool, device="cuda"))


def test_chunked_cache_reference_semantics():
    from actfold_b200.core import ChunkedActivationCache

    c = ChunkedActivationCache(max_entries_per_layer=128, chunk_size=4, device="cuda")
    acts = {"hidden_states": torch.randn(1, 8, 16, device="cuda"), "ffn_out": torch.randn(1, 8, 16, device="cuda")}
    c.put("branch", 0, acts)
    r = c.get("branch", 0, torch.ones(1, 8, dtype=torch.bool, device="cuda"))
    torch.testing.assert_close(r["hidden_states"], acts["hidden_states"], rtol=0, atol=0)
    mask = torch.tensor([[False, True, False, True, False, False, False, False]], device="cuda")
    r = c.get("branch", 0, mask)
    torch.testing.assert_close(r["hidden_states"], acts["hidden_states"][:, [1, 3]], rtol=0, atol=0)
    d = c.get_dense("branch", 0, mask)["ffn_out"]
    assert d.shape == (1, 8, 16) and (d[:, [0, 2, 4, 5, 6, 7]] == 0).all()
    c2 = ChunkedActivationCache(max_entries_per_layer=128, chunk_size=2, device="cuda")
    c2.put("b1", 0, {"x": torch.randn(1, 4, 8, device="cuda")})
    c2.put("b2", 0, {"x": torch.randn(1, 4, 8, device="cuda")})
    c2.clear_branch("b1")
    ones = torch.ones(1, 4, dtype=torch.bool, device="cuda")
    assert c2.get("b1", 0, ones) == {} and c2.get("b2", 0, ones) != {}
    c3 = ChunkedActivationCache(max_entries_per_layer=128, chunk_size=4, device="cuda")
    c3.put("branch", 0, {"x": torch.randn(1, 10, 8, device="cuda")})
    assert c3.num_tokens() == 10 and c3.num_entries() == 3
