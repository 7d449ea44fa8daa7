"""Folded verification semantics restated in numpy (TEST INFRASTRUCTURE).

Follows actfold/core/folded_transformer.py:60-203 for a layer whose parent
activations are cached:

  * parent pass (parent_branch_id None, :100-104): run the layer, store
    ``hidden_states`` (layer input) and ``ffn_out`` (layer output);
  * child pass: gate the child's layer input against the parent's cached
    layer input (:124-148); all stable -> the parent's ``ffn_out`` (:162-179);
    none stable -> recompute (:183-186); otherwise the layer is recomputed on
    the FULL child sequence and merged row-wise with the parent output
    (:190-196).

The cache is assumed large enough to hold every parent entry (the plain
ActivationCache with max_entries_per_layer >= 2 T), so the KeyError fallbacks
of :135-141 never fire.

With a FoldingScheduler (:107-119) each layer has its own threshold
(``get_tau``), and a layer where ``should_fold`` is False recomputes the
whole child sequence without gating (no stable mask is recorded for it).
"""

from __future__ import annotations

from typing import Callable

import numpy as np

from oracle import llada as L
from oracle.gate import gate as gate_fn
from oracle.rows import merge


def folded_layer(
    layer: Callable[[np.ndarray], np.ndarray],
    h_child: np.ndarray,
    parent_in: np.ndarray,
    parent_out: np.ndarray,
    tau: float,
    dtype: str,
) -> tuple[np.ndarray, np.ndarray]:
    """One folded layer for a [B, T, H] child batch; parent tensors broadcast over B.

    Returns (output, stable_mask [B, T]).
    """
    B = h_child.shape[0]
    pin = np.broadcast_to(parent_in, h_child.shape)
    pout = np.broadcast_to(parent_out, h_child.shape)
    stable = gate_fn(h_child, pin, tau, "cosine", 1e-8, dtype).mask
    if stable.all():
        return np.array(pout), stable
    full = np.stack([layer(h_child[b]) for b in range(B)])
    if not stable.any():
        return full, stable
    return merge(pout, full, stable), stable


def llada_parent(tokens: np.ndarray, weights: dict, dims: L.LLaDADims) -> dict:
    """Parent pass: per-layer inputs [L+1, T, H], K/V [L, T, Hkv] and logits [T, V]."""
    return L.dense_forward(tokens, weights, dims)


def llada_folded_children(
    children: np.ndarray,
    parent: dict,
    weights: dict,
    dims: L.LLaDADims,
    tau: float,
    layer_taus=None,
    layer_folds=None,
) -> dict:
    """Verify each child [C, T] against the cached parent, sequentially (as the reference does).

    Returns masks [L, C, T] (True = stable; all False on a layer that does not
    fold), per-layer child states [L+1, C, T, H] and logits [C, T, V].
    ``layer_taus`` / ``layer_folds``: the per-layer schedule (default: ``tau``
    and folding on every layer).
    """
    C, T = children.shape
    taus = list(layer_taus) if layer_taus is not None else [tau] * dims.n_layers
    folds = list(layer_folds) if layer_folds is not None else [True] * dims.n_layers
    cos, sin = L.rope_tables(T, dims.head_dim, dims.rope_theta)
    masks = np.zeros((dims.n_layers, C, T), bool)
    states = np.zeros((dims.n_layers + 1, C, T, dims.hidden), np.float32)
    logits = np.zeros((C, T, dims.vocab), np.float32)
    for c in range(C):
        h = weights["embed"][children[c]][None]
        states[0, c] = h[0]
        for li, lw in enumerate(weights["layers"]):
            layer = lambda x, lw=lw: L.block(x, lw, dims, cos, sin)  # noqa: E731
            if folds[li]:
                h, m = folded_layer(layer, h, parent["layer_in"][li][None], parent["layer_in"][li + 1][None], taus[li], "bf16")
                masks[li, c] = m[0]
            else:
                h = layer(h[0])[None]
            states[li + 1, c] = h[0]
        logits[c] = L.lm_head(h[0], weights, dims)
    return {"masks": masks, "states": states, "logits": logits}


def llada_promote(folded: dict, c: int) -> dict:
    """Child ``c`` of a folded result as a parent (TEST INFRASTRUCTURE).

    The reference stores a verified child's merged per-layer states under its
    own branch id (actfold/core/folded_transformer.py:190-199, :260-274), so a
    later child that names it as parent_branch_id is gated against those
    states and takes their outputs on stable rows.
    """
    return {"layer_in": np.ascontiguousarray(folded["states"][:, c]), "logits": np.ascontiguousarray(folded["logits"][c])}


def llada_resize_parent(parent: dict, T: int) -> dict:
    """The parent's cached rows for a child of length ``T`` (TEST INFRASTRUCTURE).

    The reference gathers the parent's entry of every child position and
    zero-fills positions the parent has no entry for
    (actfold/core/fused_ops.py:54-87, 256-324): rows past the parent's length
    are zeros; a shorter child sees the parent's first ``T`` rows.
    """
    out = {}
    for k in ("layer_in", "logits"):
        a = parent[k]
        ax = a.ndim - 2  # the position axis
        n = min(T, a.shape[ax])
        shape = list(a.shape)
        shape[ax] = T
        b = np.zeros(shape, a.dtype)
        idx = [slice(None)] * a.ndim
        idx[ax] = slice(0, n)
        b[tuple(idx)] = a[tuple(idx)]
        out[k] = b
    return out
