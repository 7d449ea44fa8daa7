"""FoldedTransformerLayer: the per-layer fold decision for an arbitrary layer module.

Drop-in for actfold/core/folded_transformer.py:23-274: the same constructor
and ``forward`` signature, and the same observable decisions -- the branch
context (explicit arguments, else FOLDING_CONTEXT), the scheduler's
should_fold / get_tau, a full recompute when there is no parent, the parent's
rows are missing (KeyError / RuntimeError) or no row is stable, the parent's
output when every row is stable, a merge otherwise (a missing parent output is
a RuntimeError there), the first element of tuple outputs, keyword arguments
filtered to what the wrapped layer accepts, and the child's input and output
stored afterwards. This is the GENERIC path: the wrapped layer is user code and runs
on all rows, exactly as in the reference; around it the gate, merge and cache
traffic run on the CUDA kernels:

* the parent's cached input feeds ``af_gate`` straight from the cache block
  (no zero-filled copy, parent rows broadcast over the child batch);
* the gate's fused compaction yields the divergent count, read with ONE
  host synchronisation per layer (the reference synchronises at least three
  times: ``.item()`` in the profiler, ``.all()``, ``.any()``);
* the merge reads the parent's cached output block directly.

LLaDA-architecture models wrapped by FoldedModel do not come through here:
they run the native batched pass that recomputes only divergent rows
(actfold_b200.llada).
"""

from __future__ import annotations

import inspect
from typing import Any

import torch
import torch.nn as nn

from actfold_b200.core.folding_context import FOLDING_CONTEXT
from actfold_b200.core.folding_scheduler import FoldingScheduler
from actfold_b200.core.fused_ops import merge_stable_divergent
from actfold_b200.core.similarity_gate import SimilarityGate
from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER

_BRANCH_KEYS = frozenset({"branch_id", "parent_branch_id", "step_idx"})


def _dense_get(cache, branch_id, layer_idx, token_mask):
    """Zero-filled full-shape get for either cache type (ActivationCache contract)."""
    if hasattr(cache, "get_dense"):
        return cache.get_dense(branch_id, layer_idx, token_mask)
    return cache.get(branch_id, layer_idx, token_mask)


class _LayerCall:
    """How to call a wrapped layer: which keyword arguments it takes (its signature, read once)."""

    def __init__(self, layer: nn.Module) -> None:
        params = inspect.signature(layer.forward).parameters
        self.names = frozenset(params)
        self.any_kw = any(p.kind == inspect.Parameter.VAR_KEYWORD for p in params.values())

    def __call__(self, layer: nn.Module, x: torch.Tensor, attention_mask, kwargs: dict) -> torch.Tensor:
        kw = {k: v for k, v in kwargs.items() if k not in _BRANCH_KEYS and (self.any_kw or k in self.names)}
        if attention_mask is not None and "attention_mask" in self.names:
            kw["attention_mask"] = attention_mask
        out = layer(x, **kw)
        return out[0] if isinstance(out, tuple) else out  # (hidden_states, ...) layers: the first element


class FoldedTransformerLayer(nn.Module):
    def __init__(
        self,
        original_layer: nn.Module,
        cache,
        gate: SimilarityGate,
        layer_idx: int,
        scheduler: FoldingScheduler | None = None,
    ) -> None:
        super().__init__()
        self.original_layer = original_layer
        self.cache = cache
        self.gate = gate
        self.layer_idx = layer_idx
        self.scheduler = scheduler
        self._call: _LayerCall | None = None

    def forward(
        self,
        hidden_states: torch.Tensor,
        branch_id: str | None = None,
        parent_branch_id: str | None = None,
        attention_mask: torch.Tensor | None = None,
        step_idx: int = 0,
        **kwargs: Any,
    ) -> torch.Tensor:
        if branch_id is None:  # explicit arguments win over the folding context
            ctx = FOLDING_CONTEXT.get() or {}
            branch_id = ctx.get("branch_id")
            if branch_id is not None:
                parent_branch_id = ctx.get("parent_branch_id", parent_branch_id)
                step_idx = ctx.get("step_idx", step_idx)
        if branch_id is None:
            raise ValueError(
                "FoldedTransformerLayer requires a branch_id either as an argument or via the ActFold folding context."
            )
        out = None
        if parent_branch_id is not None and self._folds_at(step_idx):
            out = self._fold(hidden_states, branch_id, parent_branch_id, step_idx, attention_mask, kwargs)
        if out is None:  # no parent, an unfolded layer, parent rows missing, or nothing stable
            out = self._run_layer(hidden_states, attention_mask, kwargs)
        self.cache.put(branch_id=branch_id, layer_idx=self.layer_idx,
                       activations={"ffn_out": out, "hidden_states": hidden_states})
        return out

    def _folds_at(self, step_idx: int) -> bool:
        """Scheduler decision for this layer; sets the shared gate's tau when the layer folds."""
        if self.scheduler is None:
            return True
        if not self.scheduler.should_fold(self.layer_idx, step_idx):
            return False
        self.gate.set_tau(self.scheduler.get_tau(layer_idx=self.layer_idx, step_idx=step_idx, task_type="general"))
        return True

    def _parent_rows(self, parent_branch_id, name: str, B: int, T: int, device, any_stable=None):
        """The parent's cached ``name`` rows for this layer; None when the cache has none."""
        rows = self.cache.dense_rows(parent_branch_id, self.layer_idx, name, T)
        if rows is not None:
            self.cache.touch(parent_branch_id, self.layer_idx, any_stable, T)
            return rows.expand(B, *rows.shape[1:]) if rows.shape[0] == 1 and B > 1 else rows
        mask = torch.ones((B, T), dtype=torch.bool, device=device) if any_stable is None else any_stable
        return _dense_get(self.cache, parent_branch_id, self.layer_idx, mask).get(name)

    def _fold(self, hidden_states, branch_id, parent_branch_id, step_idx, attention_mask, kwargs):
        """The folded output, or None when the layer has to be recomputed on every row."""
        B, T = hidden_states.shape[:2]
        try:
            h_parent = self._parent_rows(parent_branch_id, "hidden_states", B, T, hidden_states.device)
        except (KeyError, RuntimeError):
            return None
        if h_parent is None:
            return None
        g = self.gate.forward_compact(hidden_states, h_parent.to(dtype=hidden_states.dtype, device=hidden_states.device))
        stable = g.stable_mask
        GLOBAL_STABILITY_PROFILER.record(branch_id=branch_id, parent_branch_id=parent_branch_id, layer_idx=self.layer_idx,
                                         step_idx=step_idx, stable_mask=stable, tau=self.gate.tau, metric=self.gate.metric)
        # One host read per layer: the divergent total and, per position, whether any row keeps the parent's.
        host = torch.cat([g.div_count.sum().view(1), stable.any(dim=0).to(torch.int32)]).cpu().numpy()
        n_div, any_stable = int(host[0]), host[1:].astype(bool)
        if n_div == B * T:
            return None
        if n_div == 0:
            try:
                return _dense_get(self.cache, parent_branch_id, self.layer_idx, stable).get("ffn_out")
            except (KeyError, RuntimeError):
                return None
        parent_out = self.cache.dense_rows(parent_branch_id, self.layer_idx, "ffn_out", T)
        if parent_out is not None:
            self.cache.touch(parent_branch_id, self.layer_idx, any_stable, T)
        else:  # a missing parent output here is an error, as in the reference's merge path
            parent_out = _dense_get(self.cache, parent_branch_id, self.layer_idx, stable).get("ffn_out")
            if parent_out is None:
                raise RuntimeError(f"Parent FFN output missing for branch={parent_branch_id}, layer={self.layer_idx}")
        fresh = self._run_layer(hidden_states, attention_mask, kwargs)
        if parent_out.shape[0] == 1 and B > 1:
            parent_out = parent_out.expand(B, *parent_out.shape[1:])
        return merge_stable_divergent(parent_out, fresh, stable)

    def _run_layer(self, hidden_states: torch.Tensor, attention_mask, kwargs: dict) -> torch.Tensor:
        if self._call is None:
            self._call = _LayerCall(self.original_layer)
        return self._call(self.original_layer, hidden_states, attention_mask, kwargs)
