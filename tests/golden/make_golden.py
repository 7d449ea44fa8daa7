"""Generate the golden vectors under tests/golden/ by running the REFERENCE itself.

Run from the repository root, naming the reference checkout (read-only) with
``--reference`` or the ACTFOLD_REFERENCE environment variable:

    python tests/golden/make_golden.py --reference <path to the ActFold checkout>

The reference is pure Python/PyTorch. Importing ``actfold.core`` pulls
``actfold/profiler/visualization.py``, which imports matplotlib (absent here),
so a throw-away stub package for matplotlib/seaborn is written to a temporary
directory and put on ``sys.path`` before the reference. Nothing is written
into the reference tree.

Outputs (all small, compressed):
  gate.npz       reference SimilarityGate masks + similarity bits per GATE_CASE
  merge.npz      reference merge_stable_divergent outputs (fp32/fp16/bf16)
  cache.npz      reference ActivationCache op log (puts, gets, LRU, KeyErrors)
  demo.npz       reference folded pass of demo.py's synthetic model (config 1)
  llada_tiny.npz reference FoldedModel over the restated tiny LLaDA block (bf16)
  dream_tiny.npz same, GQA (Dream-shaped) tiny model
  llada_chain.npz grandchildren folded against a verified child (chained folding)
  llada_resize.npz children longer / shorter than their parent (zero-filled parent rows)
  sched.npz      reference FoldedModel with a FoldingScheduler (per-layer tau,
                 a disabled layer, the final layer and step unfolded)
  fgen.npz       reference folded_generate (greedy steps, and drafted candidates
                 with the greedy policy) over the tiny LLaDA block
  engine.npz     reference ActFoldVerificationEngine.verify_branch over the tiny
                 LLaDA block: acceptance, stable ratio, score, per-layer profile
                 and cache clearing at two thresholds, and a chained step
"""

from __future__ import annotations

import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import torch  # noqa: E402

from actfold_b200 import workloads as W  # noqa: E402
from gen_inputs import DEMO, GATE_CASES, TINY_DREAM, TINY_ENGINE, TINY_LLADA, TINY_LLADA_CHAIN, TINY_FGEN, TINY_LLADA_RESIZE, TINY_SCHED, AppendDraft, digest, engine_children, gate_inputs  # noqa: E402
from oracle import llada as OL  # noqa: E402
from oracle.llada_torch import TorchLLaDA  # noqa: E402


def _import_reference(ref: str):
    shim = tempfile.mkdtemp(prefix="af_mpl_shim_")
    os.makedirs(os.path.join(shim, "matplotlib"))
    with open(os.path.join(shim, "matplotlib", "__init__.py"), "w") as f:
        f.write("def use(*a, **k):\n    pass\n")
    with open(os.path.join(shim, "matplotlib", "pyplot.py"), "w") as f:
        f.write("def __getattr__(name):\n    raise AttributeError(name)\n")
    os.makedirs(os.path.join(shim, "seaborn"))
    with open(os.path.join(shim, "seaborn", "__init__.py"), "w") as f:
        f.write("")
    sys.path.insert(0, ref)
    sys.path.insert(0, shim)
    import actfold.core as core  # noqa: F401

    return core


TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def make_gate(core) -> None:
    out = {}
    for name, seed, B, T, H, dt, tau, metric in GATE_CASES:
        c, p = gate_inputs(seed, B, T, H, dt)
        tc = torch.from_numpy(c).to(TORCH_DT[dt])
        tp = torch.from_numpy(p).to(TORCH_DT[dt])
        g = core.SimilarityGate(tau=tau, metric=metric)
        with torch.no_grad():
            mask = g(tc, tp)
            sim = g._compute_similarity(tc, tp)
        out[f"{name}/mask"] = mask.numpy()
        if dt == "f32":
            out[f"{name}/sim"] = sim.numpy()
        else:
            out[f"{name}/sim_bits"] = sim.view(torch.int16).numpy().view(np.uint16)
        out[f"{name}/digest"] = np.array(digest(c, p))
    np.savez_compressed(os.path.join(HERE, "gate.npz"), **out)


def make_merge(core) -> None:
    from actfold.core.fused_ops import merge_stable_divergent

    out = {}
    g = torch.Generator().manual_seed(5)
    for dt in ("f32", "f16", "bf16"):
        p = torch.randn(2, 8, 64, generator=g).to(TORCH_DT[dt])
        c = torch.randn(2, 8, 64, generator=g).to(TORCH_DT[dt])
        m = torch.rand(2, 8, generator=g) > 0.5
        o = merge_stable_divergent(p, c, m)
        out[f"{dt}/parent"] = p.float().numpy()
        out[f"{dt}/child"] = c.float().numpy()
        out[f"{dt}/mask"] = m.numpy()
        out[f"{dt}/out"] = o.float().numpy()
    np.savez_compressed(os.path.join(HERE, "merge.npz"), **out)


def cache_script():
    """A fixed op sequence exercising put/get/LRU/touch/clear/step keys (shared with the tests)."""
    g = torch.Generator().manual_seed(9)
    ops = []

    def acts(B, T, H, names=("ffn_out", "hidden_states")):
        return {n: torch.randn(B, T, H, generator=g) for n in names}

    ops.append(("put", "p", 0, acts(1, 6, 8), 0))
    ops.append(("get", "p", 0, torch.tensor([[True, False, True, True, False, True]]), 0))
    ops.append(("put", "c1", 0, acts(1, 6, 8), 0))
    ops.append(("get", "p", 0, torch.ones(2, 6, dtype=torch.bool), 0))  # batch broadcast
    ops.append(("put", "c2", 0, acts(1, 6, 8), 0))  # evicts c1's oldest tokens (p was touched)
    ops.append(("get", "c1", 0, torch.ones(1, 6, dtype=torch.bool), 0))
    ops.append(("get", "p", 0, torch.tensor([[False, True, False, False, True, False]]), 0))
    ops.append(("put", "c3", 0, acts(1, 4, 8), 0))  # evicts p's untouched tokens
    ops.append(("get", "p", 0, torch.ones(1, 6, dtype=torch.bool), 0))
    ops.append(("get", "c2", 0, torch.tensor([[True, True, False, True, True, True]]), 0))
    ops.append(("put", "s", 1, acts(2, 5, 4), 3))
    ops.append(("get", "s", 1, torch.tensor([[True, False, True, False, True], [False, True, True, True, False]]), 3))
    ops.append(("get", "s", 1, torch.ones(2, 5, dtype=torch.bool), 0))  # wrong step -> KeyError
    ops.append(("clear_branch", "c2"))
    ops.append(("get", "c2", 0, torch.ones(1, 6, dtype=torch.bool), 0))
    ops.append(("clear_layer", 1))
    ops.append(("put", "s", 1, {"ffn_out": torch.randn(1, 3, 4, generator=g)}, 0))
    ops.append(("get", "s", 1, torch.ones(1, 3, dtype=torch.bool), 0))
    return ops


def make_cache(core) -> None:
    cache = core.ActivationCache(max_entries_per_layer=14, device="cpu")
    out = {}
    log = []
    for i, op in enumerate(cache_script()):
        kind = op[0]
        rec = {"i": i, "kind": kind}
        if kind == "put":
            _, b, l, a, s = op
            rec.update(branch=b, layer=l, step=s, names=list(a))
            cache.put(b, l, a, step_idx=s)
            for n, t in a.items():
                out[f"{i}/in/{n}"] = t.numpy()
        elif kind == "get":
            _, b, l, m, s = op
            rec.update(branch=b, layer=l, step=s)
            out[f"{i}/mask"] = m.numpy()
            try:
                r = cache.get(b, l, m, step_idx=s)
                rec["out_names"] = sorted(r)
                for n, t in r.items():
                    out[f"{i}/out/{n}"] = t.numpy()
            except KeyError:
                rec["keyerror"] = True
        elif kind == "clear_branch":
            rec["branch"] = op[1]
            cache.clear_branch(op[1])
        elif kind == "clear_layer":
            rec["layer"] = op[1]
            cache.clear_layer(op[1])
        rec["num_entries"] = cache.num_entries()
        rec["num_entries_l0"] = cache.num_entries(0)
        log.append(rec)
    out["log"] = np.array(json.dumps(log))
    np.savez_compressed(os.path.join(HERE, "cache.npz"), **out)


def make_demo(core) -> None:
    sys.path.insert(0, REF)
    import demo  # reference demo.py

    from actfold.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER

    w = W.demo_weights(seed=DEMO["weight_seed"])
    parent, children = W.demo_tokens(seed=DEMO["token_seed"], T=DEMO["T"], n_children=DEMO["n_children"])
    cache = core.ActivationCache(max_entries_per_layer=1024, device="cpu")
    gate = core.SimilarityGate(tau=DEMO["tau"], metric="cosine")
    model = demo.FoldedSyntheticTransformer(1000, 128, 4, 8, cache, gate)
    base = demo.SyntheticTransformer(1000, 128, 4, 8)
    with torch.no_grad():
        for m in (model, base):
            m.embedding.weight.copy_(torch.from_numpy(w["embedding"]))
            m.lm_head.weight.copy_(torch.from_numpy(w["lm_head"]))
        for lw, fl, bl in zip(w["layers"], model.layers, base.layers):
            for tgt in (fl.original_layer, bl):
                tgt.attn.in_proj_weight.copy_(torch.from_numpy(lw["in_proj_weight"]))
                tgt.attn.in_proj_bias.copy_(torch.from_numpy(lw["in_proj_bias"]))
                tgt.attn.out_proj.weight.copy_(torch.from_numpy(lw["out_proj_weight"]))
                tgt.attn.out_proj.bias.copy_(torch.from_numpy(lw["out_proj_bias"]))
                tgt.norm1.weight.copy_(torch.from_numpy(lw["norm1_weight"]))
                tgt.norm1.bias.copy_(torch.from_numpy(lw["norm1_bias"]))
                tgt.ffn[0].weight.copy_(torch.from_numpy(lw["ffn0_weight"]))
                tgt.ffn[0].bias.copy_(torch.from_numpy(lw["ffn0_bias"]))
                tgt.ffn[2].weight.copy_(torch.from_numpy(lw["ffn2_weight"]))
                tgt.ffn[2].bias.copy_(torch.from_numpy(lw["ffn2_bias"]))
                tgt.norm2.weight.copy_(torch.from_numpy(lw["norm2_weight"]))
                tgt.norm2.bias.copy_(torch.from_numpy(lw["norm2_bias"]))
    model.eval()
    base.eval()
    GLOBAL_STABILITY_PROFILER.reset()
    out = {}
    with torch.no_grad():
        pl = model(torch.from_numpy(parent)[None], branch_id="parent")
        out["parent_logits"] = pl[0].numpy()
        masks, logits, base_logits = [], [], []
        for c in range(children.shape[0]):
            ct = torch.from_numpy(children[c])[None]
            lg = model(ct, branch_id=f"child{c}", parent_branch_id="parent")
            prof = GLOBAL_STABILITY_PROFILER.get_profile(f"child{c}")
            m = np.ones((4, DEMO["T"]), bool)
            for st in prof.layer_stats:
                if st.divergence_positions is not None:
                    for _, t in st.divergence_positions.tolist():
                        m[st.layer_idx, t] = False
            masks.append(m)
            logits.append(lg[0].numpy())
            base_logits.append(base(ct)[0].numpy())
    out["masks"] = np.stack(masks, axis=1)  # [L, C, T]
    out["logits"] = np.stack(logits)
    out["base_logits"] = np.stack(base_logits)
    out["parent"] = parent
    out["children"] = children
    np.savez_compressed(os.path.join(HERE, "demo.npz"), **out)


def make_llada(core, dims: W.ModelDims, spec: dict, fname: str) -> None:
    from actfold.core.model_wrapper import FoldedModel

    od = OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab, dims.rms_eps, dims.rope_theta)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    T = spec["T"]
    parent, children = W.llada_tokens(T, spec["n_prompt"], spec["mask_frac"], spec["n_children"], spec["d"], dims.mask_id, spec["token_seed"])
    C = children.shape[0]
    model = TorchLLaDA(w, od, T)
    cache = core.ActivationCache(max_entries_per_layer=(C + 2) * T, device="cpu")
    gate = core.SimilarityGate(tau=spec["tau"], metric="cosine")
    folded = FoldedModel(model, cache, gate)
    assert folded.folding_applied
    recorded: list = []
    orig_forward = gate.forward

    def rec_forward(hc, hp):
        m = orig_forward(hc, hp)
        recorded.append(m.clone())
        return m

    gate.forward = rec_forward  # instance attribute; nn.Module.__call__ dispatches to it
    states: list = []
    hooks = [layer.register_forward_hook(lambda mod, inp, outp: states.append(outp.clone())) for layer in folded.wrapped_model.layers]
    out = {}
    with torch.no_grad():
        pl = folded(torch.from_numpy(parent)[None], branch_id="parent")
        out["parent_logits_bits"] = pl[0].view(torch.int16).numpy().view(np.uint16)
        parent_states = [s[0] for s in states]
        states.clear()
        masks, logits, child_states = [], [], []
        for c in range(C):
            recorded.clear()
            states.clear()
            lg = folded(torch.from_numpy(children[c])[None], branch_id=f"child{c}", parent_branch_id="parent")
            masks.append(torch.stack([m[0] for m in recorded]).numpy())
            logits.append(lg[0].view(torch.int16).numpy().view(np.uint16))
            child_states.append(torch.stack([s[0] for s in states]).view(torch.int16).numpy().view(np.uint16))
    for h in hooks:
        h.remove()
    out["masks"] = np.stack(masks, axis=1)  # [L, C, T]
    out["logits_bits"] = np.stack(logits)  # [C, T, V]
    out["state_bits"] = np.stack(child_states, axis=1)  # [L, C, T, H] layer outputs
    out["parent_state_bits"] = torch.stack(parent_states).view(torch.int16).numpy().view(np.uint16)
    out["parent"] = parent
    out["children"] = children
    np.savez_compressed(os.path.join(HERE, fname), **out)


def make_llada_chain(core, dims: W.ModelDims, spec: dict, fname: str) -> None:
    """Chained folding: grandchildren verified with parent_branch_id = a verified child's id.

    The reference stores every child's activations (folded_transformer.py:190-199),
    so the grandchildren fold against the child's merged per-layer states.
    """
    from actfold.core.model_wrapper import FoldedModel

    od = OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab, dims.rms_eps, dims.rope_theta)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    T = spec["T"]
    parent, children = W.llada_tokens(T, spec["n_prompt"], spec["mask_frac"], spec["n_children"], spec["d"], dims.mask_id, spec["token_seed"])
    k = spec["chain_child"]
    grand = W.llada_children(children[k], spec["chain_n"], spec["chain_d"], dims.mask_id, spec["chain_seed"])
    model = TorchLLaDA(w, od, T)
    cache = core.ActivationCache(max_entries_per_layer=(children.shape[0] + grand.shape[0] + 2) * T, device="cpu")
    gate = core.SimilarityGate(tau=spec["tau"], metric="cosine")
    folded = FoldedModel(model, cache, gate)
    recorded: list = []
    orig_forward = gate.forward

    def rec_forward(hc, hp):
        m = orig_forward(hc, hp)
        recorded.append(m.clone())
        return m

    gate.forward = rec_forward
    out = {}
    with torch.no_grad():
        folded(torch.from_numpy(parent)[None], branch_id="parent")
        for c in range(children.shape[0]):
            folded(torch.from_numpy(children[c])[None], branch_id=f"child{c}", parent_branch_id="parent")
        masks, logits = [], []
        for g in range(grand.shape[0]):
            recorded.clear()
            lg = folded(torch.from_numpy(grand[g])[None], branch_id=f"grand{g}", parent_branch_id=f"child{k}")
            masks.append(torch.stack([m[0] for m in recorded]).numpy())
            logits.append(lg[0].view(torch.int16).numpy().view(np.uint16))
    out["masks"] = np.stack(masks, axis=1)  # [L, G, T]
    out["logits_bits"] = np.stack(logits)  # [G, T, V]
    out["parent"] = parent
    out["children"] = children
    out["chain_child"] = np.array(k)
    out["grandchildren"] = grand
    np.savez_compressed(os.path.join(HERE, fname), **out)


def make_llada_resize(core, dims: W.ModelDims, spec: dict, fname: str) -> None:
    """Children longer and shorter than their parent.

    The reference gathers the parent's entries for the child's positions and
    zero-fills the ones the parent lacks (fused_ops.py:54-87), so appended
    positions gate as divergent against zero rows while the shared prefix folds.
    """
    from actfold.core.model_wrapper import FoldedModel

    od = OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab, dims.rms_eps, dims.rope_theta)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    T, Tp, Ts = spec["T"], spec["parent_len"], spec["short_len"]
    full, _ = W.llada_tokens(T, spec["n_prompt"], spec["mask_frac"], 1, 1, dims.mask_id, spec["token_seed"])
    parent = full[:Tp].copy()
    rng = np.random.default_rng(spec["token_seed"] + 1)
    longer = np.repeat(full[None], spec["n_children"], axis=0)
    longer[:, Tp:] = rng.integers(0, dims.mask_id, size=(spec["n_children"], T - Tp))
    shorter = W.llada_children(parent[:Ts], spec["n_children"], spec["d"], dims.mask_id, spec["token_seed"] + 2)
    model = TorchLLaDA(w, od, T)
    cache = core.ActivationCache(max_entries_per_layer=(2 * spec["n_children"] + 2) * T, device="cpu")
    gate = core.SimilarityGate(tau=spec["tau"], metric="cosine")
    folded = FoldedModel(model, cache, gate)
    recorded: list = []
    orig_forward = gate.forward

    def rec_forward(hc, hp):
        m = orig_forward(hc, hp)
        recorded.append(m.clone())
        return m

    gate.forward = rec_forward
    out = {"parent": parent, "longer": longer, "shorter": shorter}
    with torch.no_grad():
        folded(torch.from_numpy(parent)[None], branch_id="parent")
        for name, kids in (("longer", longer), ("shorter", shorter)):
            masks, logits = [], []
            for c in range(kids.shape[0]):
                recorded.clear()
                lg = folded(torch.from_numpy(kids[c])[None], branch_id=f"{name}{c}", parent_branch_id="parent")
                masks.append(torch.stack([m[0] for m in recorded]).numpy())
                logits.append(lg[0].view(torch.int16).numpy().view(np.uint16))
            out[f"{name}_masks"] = np.stack(masks, axis=1)
            out[f"{name}_logits_bits"] = np.stack(logits)
    np.savez_compressed(os.path.join(HERE, fname), **out)


def make_sched(core, dims: W.ModelDims, spec: dict, fname: str) -> None:
    """FoldedModel(..., scheduler=FoldingScheduler) over the restated tiny LLaDA block.

    Per folded layer the reference sets the shared gate's tau to
    get_tau(layer, step) and records the mask; a layer where should_fold is
    False (a disabled layer, the final layer, every layer of the final step)
    recomputes without gating (actfold/core/folded_transformer.py:107-119).
    Recorded per step: the folded layers, their tau, masks, logits and the
    gate's tau after the step.
    """
    import dataclasses

    from actfold.core.folding_scheduler import FoldingScheduler
    from actfold.core.model_wrapper import FoldedModel
    from actfold.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER

    dims = dataclasses.replace(dims, n_layers=spec["n_layers"])
    od = OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab, dims.rms_eps, dims.rope_theta)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    T = spec["T"]
    parent, children = W.llada_tokens(T, spec["n_prompt"], spec["mask_frac"], spec["n_children"], spec["d"], dims.mask_id, spec["token_seed"])
    C = children.shape[0]
    model = TorchLLaDA(w, od, T)
    cache = core.ActivationCache(max_entries_per_layer=(C * len(spec["steps"]) + 2) * T, device="cpu")
    gate = core.SimilarityGate(tau=spec["tau"], metric="cosine")
    sched = FoldingScheduler(base_tau=spec["tau"], num_layers=dims.n_layers, num_steps=spec["num_steps"],
                             disabled_layers=set(spec["disabled_layers"]))
    folded = FoldedModel(model, cache, gate, scheduler=sched)
    out = {"parent": parent, "children": children}
    with torch.no_grad():
        folded(torch.from_numpy(parent)[None], branch_id="parent")
        for step in spec["steps"]:
            masks, taus, layers, logits = [], [], None, []
            for c in range(C):
                bid = f"s{step}c{c}"
                GLOBAL_STABILITY_PROFILER.reset_branch(bid)
                lg = folded(torch.from_numpy(children[c])[None], branch_id=bid, parent_branch_id="parent", step_idx=step)
                prof = GLOBAL_STABILITY_PROFILER.get_profile(bid)
                stats = prof.layer_stats if prof is not None else []
                ls = [st.layer_idx for st in stats]
                assert layers is None or layers == ls
                layers = ls
                taus = [st.tau_used for st in stats]
                m = np.zeros((len(ls), T), bool)
                for i, st in enumerate(stats):
                    if st.divergence_positions is not None:
                        m[i] = True
                        m[i, st.divergence_positions[:, 1].numpy()] = False
                    else:
                        m[i] = True
                masks.append(m)
                logits.append(lg[0].view(torch.int16).numpy().view(np.uint16))
            out[f"step{step}/layers"] = np.array(layers, np.int64)
            out[f"step{step}/taus"] = np.array(taus, np.float64)
            out[f"step{step}/masks"] = np.stack(masks, axis=1) if layers else np.zeros((0, C, T), bool)
            out[f"step{step}/logits_bits"] = np.stack(logits)
            out[f"step{step}/gate_tau_after"] = np.array(gate.tau)
    np.savez_compressed(os.path.join(HERE, fname), **out)


def make_fgen(core, dims: W.ModelDims, spec: dict, fname: str) -> None:
    """The reference folded_generate (actfold/speculative/folded_generation.py:44-238) over FoldedModel.

    Greedy mode: each step appends the argmax of the accepted sequence's last
    logits and folds the child against it. Draft mode: AppendDraft proposes
    n_branches one-id extensions per step, each folded against the accepted
    sequence, GreedyAcceptancePolicy keeps the one with the largest
    last-position logit. Recorded: the accepted tokens after every step, the
    accepted node's stable ratio, the greedy top-2 margins (greedy mode) and
    every candidate's score (draft mode), and the final result fields.
    """
    import torch.nn as nn
    from actfold.core.model_wrapper import FoldedModel
    from actfold.speculative.acceptance_policy import GreedyAcceptancePolicy
    from actfold.speculative.fast_dllm_adapter import FastDLLMAdapter
    from actfold.speculative.folded_generation import folded_generate

    od = OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab, dims.rms_eps, dims.rope_theta)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    Tmax = spec["T"] + spec["max_new_tokens"]

    class Emb(nn.Module):
        def __init__(self, table):
            super().__init__()
            self.table = table

        def forward(self, tokens):
            return self.table[tokens]

    class Recording(GreedyAcceptancePolicy):
        def __init__(self):
            self.scores = []

        def select(self, candidates, logits=None):
            self.scores.append([float(n.logits[:, -1, :].max(dim=-1).values.mean()) for n in candidates])
            return super().select(candidates, logits)

    def run(prompt, draft):
        model = TorchLLaDA(w, od, Tmax)
        model.embedding = Emb(model.embed)
        cache = core.ActivationCache(max_entries_per_layer=64 * Tmax, device="cpu")
        gate = core.SimilarityGate(tau=spec["tau"], metric="cosine")
        folded = FoldedModel(model, cache, gate)
        adapter = FastDLLMAdapter(folded.wrapped_model, num_layers=dims.n_layers, hidden_dim=dims.hidden,
                                  num_heads=dims.n_heads, vocab_size=dims.vocab, folded_model=folded)
        pol = Recording()
        steps = []
        orig = pol.select

        def select(cands, logits=None):
            chosen = orig(cands, logits)
            steps.append((chosen.tokens[0].clone(), float(chosen.metadata.get("stable_ratio", -1.0)),
                          [n.tokens[0].clone() for n in cands]))
            return chosen

        pol.select = select
        with torch.no_grad():
            res = folded_generate(adapter, prompt, spec["max_new_tokens"], folded_model=folded,
                                  draft_generator=draft, acceptance_policy=pol,
                                  num_branches_per_step=spec["n_branches"] if draft is not None else 1)
        return res, steps, pol.scores

    def greedy_margins(prompt, steps):
        # top-2 margin of the last logits of each accepted sequence that a greedy step extended
        model = TorchLLaDA(w, od, Tmax)
        seqs = [prompt[0]] + [st[0] for st in steps[:-1]]
        out = []
        with torch.no_grad():
            for sq in seqs:
                lg = model(sq[None])[0, -1].float()
                top = lg.topk(2).values
                out.append(float(top[0] - top[1]))
        return out

    seed = spec["prompt_seed"]
    while True:
        prompt = torch.from_numpy(np.random.default_rng(seed).integers(0, dims.mask_id, size=(1, spec["T"])))
        res_g, steps_g, _ = run(prompt, None)
        margins = greedy_margins(prompt, steps_g)
        if min(margins) >= spec["min_margin"]:
            break
        seed += 1
    res_d, steps_d, scores_d = run(prompt, AppendDraft(dims.mask_id))
    out = {"prompt": prompt.numpy(), "prompt_seed": np.array(seed), "greedy/margins": np.array(margins)}
    for name, res, steps in (("greedy", res_g, steps_g), ("draft", res_d, steps_d)):
        out[f"{name}/tokens"] = res.tokens.numpy()
        out[f"{name}/stable_ratio"] = np.array(res.stable_ratio)
        out[f"{name}/num_folded_steps"] = np.array(res.num_folded_steps)
        out[f"{name}/final_branch_id"] = np.array(str(res.final_branch_id))
        out[f"{name}/step_ratio"] = np.array([st[1] for st in steps])
        for i, st in enumerate(steps):
            out[f"{name}/step{i}/tokens"] = st[0].numpy()
            out[f"{name}/step{i}/candidates"] = np.stack([c.numpy() for c in st[2]])
    out["draft/scores"] = np.array(scores_d)
    np.savez_compressed(os.path.join(HERE, fname), **out)


def make_engine(core, dims: W.ModelDims, spec: dict, fname: str) -> None:
    """The reference verification engine over FoldedModel(restated tiny LLaDA).

    verify_branch (actfold/speculative/verification_engine.py:75-144) re-runs
    the parent pass, folds the child, takes the profile's mean stable ratio,
    sets metadata["actfold_score"] = mean of the child's logits and
    metadata["stable_ratio"], accepts when stable_ratio >= threshold and
    clears a rejected child's cache entries. Recorded per threshold and child:
    accepted, stable ratio, score, per-layer stable ratios and whether the
    child still has cache entries; then grandchildren of the first accepted
    child (threshold 0) verified with ``verify_branch(child, grandchild)``.
    """
    import torch.nn as nn
    from actfold.core.model_wrapper import FoldedModel
    from actfold.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER
    from actfold.speculative.branch import Branch
    from actfold.speculative.fast_dllm_adapter import FastDLLMAdapter
    from actfold.speculative.verification_engine import ActFoldVerificationEngine

    od = OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab, dims.rms_eps, dims.rope_theta)
    w = W.llada_weights_numpy(dims, seed=spec["weight_seed"])
    T = spec["T"]
    parent, _ = W.llada_tokens(T, spec["n_prompt"], spec["mask_frac"], 1, 1, dims.mask_id, spec["token_seed"])
    children = engine_children(parent, dims.mask_id, spec)
    C = children.shape[0]

    class Emb(nn.Module):
        def __init__(self, table):
            super().__init__()
            self.table = table

        def forward(self, tokens):
            return self.table[tokens]

    def run(threshold: float, chain: np.ndarray | None = None):
        model = TorchLLaDA(w, od, T)
        model.embedding = Emb(model.embed)  # the adapter looks the input embeddings up here
        cache = core.ActivationCache(max_entries_per_layer=(C + 4) * T, device="cpu")
        gate = core.SimilarityGate(tau=spec["tau"], metric="cosine")
        folded = FoldedModel(model, cache, gate)
        adapter = FastDLLMAdapter(folded.wrapped_model, num_layers=dims.n_layers, hidden_dim=dims.hidden,
                                  num_heads=dims.n_heads, vocab_size=dims.vocab, folded_model=folded)
        engine = ActFoldVerificationEngine(adapter, cache, gate, acceptance_threshold=threshold)
        pb = Branch("parent", None, torch.from_numpy(parent)[None])
        rec = {"accepted": [], "ratio": [], "score": [], "layer_ratio": [], "cached": []}
        with torch.no_grad():
            for c in range(C):
                cb = Branch(f"child{c}", "parent", torch.from_numpy(children[c])[None])
                r = engine.verify_branch(pb, cb)
                assert r.accepted == cb.accepted and cb.metadata["stable_ratio"] == r.stable_ratio
                rec["accepted"].append(bool(r.accepted))
                rec["ratio"].append(float(r.stable_ratio))
                rec["score"].append(float(cb.metadata["actfold_score"]))
                prof = GLOBAL_STABILITY_PROFILER.get_profile(f"child{c}")
                rec["layer_ratio"].append([s.stable_ratio for s in prof.layer_stats])
                rec["cached"].append(any(k[0] == f"child{c}" for lc in cache._caches.values() for k in lc))
            grand = {"ratio": [], "score": [], "layer_ratio": []}
            if chain is not None:
                k = rec["accepted"].index(True)
                kb = Branch(f"child{k}", "parent", torch.from_numpy(children[k])[None])
                for g in range(chain.shape[0]):
                    # verify_branch re-runs the dense pass of its parent branch (here the
                    # accepted child, whose cached entries it replaces) before folding.
                    gb = Branch(f"grand{g}", f"child{k}", torch.from_numpy(chain[g])[None])
                    r = engine.verify_branch(kb, gb)
                    prof = GLOBAL_STABILITY_PROFILER.get_profile(gb.branch_id)
                    grand["ratio"].append(float(r.stable_ratio))
                    grand["score"].append(float(gb.metadata["actfold_score"]))
                    grand["layer_ratio"].append([s.stable_ratio for s in prof.layer_stats])
                grand["child"] = k
        return rec, grand

    out = {"parent": parent, "children": children}
    first, _ = run(0.0)
    ratios = sorted(set(first["ratio"]))
    thr = (ratios[0] + ratios[1]) / 2 if len(ratios) > 1 else ratios[0]
    grand_tokens = None
    for name, t in (("t0", 0.0), ("t1", thr)):
        if name == "t0":
            k = 0
            grand_tokens = W.llada_children(children[k], spec["chain_n"], spec["chain_d"], dims.mask_id, spec["chain_seed"])
        rec, grand = run(t, grand_tokens if name == "t0" else None)
        out[f"{name}/threshold"] = np.array(t)
        for key, v in rec.items():
            out[f"{name}/{key}"] = np.array(v)
        if name == "t0":
            out["grand/child"] = np.array(grand["child"])
            out["grand/tokens"] = grand_tokens
            for key in ("ratio", "score", "layer_ratio"):
                out[f"grand/{key}"] = np.array(grand[key])
    np.savez_compressed(os.path.join(HERE, fname), **out)


def main() -> None:
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ACTFOLD_REFERENCE"),
                    help="path of the ActFold checkout (default: $ACTFOLD_REFERENCE)")
    ap.add_argument("--only", default=None, help="write only this fixture (e.g. engine)")
    a = ap.parse_args()
    if not a.reference or not os.path.isdir(os.path.join(a.reference, "actfold")):
        raise SystemExit("make_golden: pass --reference <ActFold checkout> (or set ACTFOLD_REFERENCE)")
    torch.manual_seed(42)
    core = _import_reference(a.reference)
    jobs = {
        "gate": lambda: make_gate(core),
        "merge": lambda: make_merge(core),
        "cache": lambda: make_cache(core),
        "demo": lambda: make_demo(core),
        "llada_tiny": lambda: make_llada(core, W.LLADA_TINY, TINY_LLADA, "llada_tiny.npz"),
        "dream_tiny": lambda: make_llada(core, W.DREAM_TINY, TINY_DREAM, "dream_tiny.npz"),
        "llada_chain": lambda: make_llada_chain(core, W.LLADA_TINY, TINY_LLADA_CHAIN, "llada_chain.npz"),
        "llada_resize": lambda: make_llada_resize(core, W.LLADA_TINY, TINY_LLADA_RESIZE, "llada_resize.npz"),
        "engine": lambda: make_engine(core, W.LLADA_TINY, TINY_ENGINE, "engine.npz"),
        "sched": lambda: make_sched(core, W.LLADA_TINY, TINY_SCHED, "sched.npz"),
        "fgen": lambda: make_fgen(core, W.LLADA_TINY, TINY_FGEN, "fgen.npz"),
    }
    for name, job in jobs.items():
        if a.only in (None, name):
            job()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
