"""Checks of a folded pass at full model size, shared by the full-size GPU tests.

The numpy oracle is too slow at LLaDA-8B / Dream-7B size, so a full-size pass
is checked layer by layer against the fp32 torch restatement of the block
(``oracle.llada_torch``: fp32 arithmetic with the oracle's bf16 rounding
points) applied on the GPU to the child's full materialised layer input, and
through size-independent properties of folding:

* the pass's stable masks equal ``SimilarityGate`` (bit-exact against the
  reference's gate on its golden vectors) applied to the materialised child
  inputs and the parent's cached inputs, at every layer;
* at layer 0 the divergent rows are exactly the edited tokens (plus the rows
  the parent fails its own gate on), and the divergent set never grows;
* stable rows of every layer's output and of the logits are bit-identical to
  the parent's;
* divergent rows of every layer's output: max relative error <= 2e-2 of the
  rows' scale and cosine >= 0.999 against the fp32 block;
* divergent rows of the final logits against an fp32 RMSNorm + LM head on the
  last layer's output rows: max relative error <= 2e-2, cosine >= 0.999 and
  argmax agreement >= 99.9 % over the rows whose argmax is defined (top-2
  margin above two bf16 ulps of the row's scale).
"""

from __future__ import annotations

import math

import torch

from oracle import llada as OL
from oracle.llada_torch import TorchLLaDABlock, _rms

REL_TOL = 2e-2
COS_TOL = 0.999
ARGMAX_TOL = 0.999


def untile(t: torch.Tensor) -> torch.Tensor:
    """[n/128, k/64, 128, 64] tiled weights -> row-major [n, k]."""
    nb, kb, r, c = t.shape
    return t.permute(0, 2, 1, 3).reshape(nb * r, kb * c)


def oracle_dims(dims) -> OL.LLaDADims:
    return OL.LLaDADims(dims.n_layers, dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.ffn, dims.vocab,
                        dims.rms_eps, dims.rope_theta)


def torch_block(model, layer: int) -> TorchLLaDABlock:
    """The fp32 restatement of block ``layer`` over the model's own (untiled) bf16 weights."""
    dims = model.dims
    blk = model.layers[layer]
    q, kv = dims.q_dim, dims.kv_dim
    wqkv = untile(blk.w_qkv)
    gu = untile(blk.w_gateup).view(dims.ffn // 64, 2, 64, dims.hidden)
    return TorchLLaDABlock.from_tensors(
        dict(attn_norm=blk.attn_norm, ffn_norm=blk.ffn_norm, wq=wqkv[:q], wk=wqkv[q:q + kv], wv=wqkv[q + kv:],
             wo=untile(blk.w_o), w_gate=gu[:, 0].reshape(dims.ffn, dims.hidden),
             w_up=gu[:, 1].reshape(dims.ffn, dims.hidden), w_down=untile(blk.w_down)),
        oracle_dims(dims), model.rope_cos, model.rope_sin)


def rel_cos(got: torch.Tensor, want: torch.Tensor) -> tuple[float, float]:
    got, want = got.double(), want.double()
    rel = float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))
    cos = float((got * want).sum() / math.sqrt(float((got * got).sum()) * float((want * want).sum())))
    return rel, cos


def argmax_stats(got: torch.Tensor, ref: torch.Tensor) -> tuple[int, int]:
    """(rows with a defined reference argmax, of those the rows whose argmax agrees)."""
    ref = ref.float()
    top2 = ref.topk(2, dim=-1).values
    scale = ref.abs().amax(-1).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(scale)) - 7)
    defined = (top2[:, 0] - top2[:, 1]) > 2 * ulp
    agree = (got.float().argmax(-1) == ref.argmax(-1)) & defined
    return int(defined.sum()), int(agree.sum())


def check_folded_pass(model, pc, parent_tokens, child_tokens, tau: float, logits: torch.Tensor, plan,
                      layers=None, children=None) -> dict:
    """Run every check of the module docstring; returns the worst figures seen."""
    from actfold_b200.core import SimilarityGate

    dims = model.dims
    L = dims.n_layers
    C = child_tokens.shape[0]
    layers = range(L) if layers is None else layers
    children = range(C) if children is None else children
    masks = plan.stable_masks()
    stats = {"layer_rel": 0.0, "layer_cos": 1.0, "logit_rel": 0.0, "logit_cos": 1.0, "defined": 0, "agree": 0,
             "div_rows": int((~masks[0]).sum())}

    # Layer 0: the edited tokens, plus rows the parent fails its own gate on.
    edited = torch.as_tensor(child_tokens != parent_tokens[None], device=masks.device)
    self_unstable = (pc.self_stable[0] == 0)[None].expand_as(edited)
    assert torch.equal(~masks[0], edited | self_unstable), "layer-0 divergent rows are not the edited tokens"
    div = ~masks
    assert not (div[1:] & ~div[:-1] & (pc.self_stable[1:] != 0)[:, None, :]).any(), "the divergent set grew"

    gate = SimilarityGate(tau=tau)
    for layer in layers:
        x = plan.materialize(layer)
        y = plan.materialize(layer + 1)
        g = gate(x, pc.layer_in[layer][None].expand_as(x))
        assert torch.equal(g, masks[layer]), f"gate decisions differ at layer {layer}"
        tb = torch_block(model, layer)
        stable_next = pc.layer_in[layer + 1]
        for c in children:
            dv = ~masks[layer, c]
            assert torch.equal(y[c][~dv], stable_next[~dv]), f"stable rows differ from the parent (layer {layer}, child {c})"
            if not dv.any():
                continue
            with torch.no_grad():
                ref = tb(x[c][None])[0]
            rel, cos = rel_cos(y[c][dv].float(), ref[dv].float())
            assert rel <= REL_TOL and cos >= COS_TOL, (layer, c, rel, cos)
            stats["layer_rel"] = max(stats["layer_rel"], rel)
            stats["layer_cos"] = min(stats["layer_cos"], cos)
        del tb

    # Final logits: stable rows are the parent's; divergent rows against fp32 norm + LM head.
    final_stable = masks[-1]
    assert torch.equal(logits[final_stable], pc.logits[None].expand_as(logits)[final_stable]), "stable logits differ"
    xf = plan.materialize(L)
    w_lm = untile(model.lm_head)
    got_rows, ref_rows = [], []
    for c in children:
        dv = ~final_stable[c]
        if not dv.any():
            continue
        a = _rms(xf[c][dv], model.final_norm, dims.rms_eps)
        with torch.no_grad():
            ref = (a.float() @ w_lm.float().T).to(torch.bfloat16)
        got_rows.append(logits[c][dv])
        ref_rows.append(ref)
    if got_rows:
        got, ref = torch.cat(got_rows), torch.cat(ref_rows)
        rel, cos = rel_cos(got.float(), ref.float())
        assert rel <= REL_TOL and cos >= COS_TOL, ("logits", rel, cos)
        stats["logit_rel"], stats["logit_cos"] = rel, cos
        stats["defined"], stats["agree"] = argmax_stats(got, ref)
        assert stats["defined"] >= 0.5 * got.shape[0], "too few rows with a defined argmax to judge"
        assert stats["agree"] >= ARGMAX_TOL * stats["defined"], ("argmax", stats["agree"], stats["defined"])
    return stats
