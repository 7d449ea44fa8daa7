"""FoldedTransformerLayer: the per-layer fold decision for an arbitrary layer module.

Drop-in for actfold/core/folded_transformer.py:23-274 (same constructor,
``forward`` signature, branch-context resolution, scheduler handling,
KeyError/RuntimeError -> recompute fallbacks, tuple outputs and kwargs
filtering). This is the GENERIC path: the wrapped layer is user code and runs
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

import numpy as np
import torch
import torch.nn as nn

from actfold_b200.core.folding_context import FOLDING_CONTEXT
from actfold_b200.core.folding_scheduler import FoldingScheduler
from actfold_b200.core.fused_ops import merge_stable_divergent
from actfold_b200.core.similarity_gate import SimilarityGate
from actfold_b200.profiler.stability_profiler import GLOBAL_STABILITY_PROFILER

_ACTFOLD_KWARGS = {"branch_id", "parent_branch_id", "step_idx"}


def _dense_get(cache, branch_id, layer_idx, token_mask):
    """Zero-filled full-shape get for either cache type (ActivationCache contract)."""
    if hasattr(cache, "get_dense"):
        return cache.get_dense(branch_id, layer_idx, token_mask)
    return cache.get(branch_id, layer_idx, token_mask)


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

    def forward(
        self,
        hidden_states: torch.Tensor,
        branch_id: str | None = None,
        parent_branch_id: str | None = None,
        attention_mask: torch.Tensor | None = None,
        step_idx: int = 0,
        **kwargs: Any,
    ) -> torch.Tensor:
        if branch_id is None:
            ctx = FOLDING_CONTEXT.get()
            if ctx is not None:
                branch_id = ctx["branch_id"]
                parent_branch_id = ctx.get("parent_branch_id", parent_branch_id)
                step_idx = ctx.get("step_idx", step_idx)
        if branch_id is None:
            raise ValueError(
                "FoldedTransformerLayer requires a branch_id either as an argument or via the ActFold folding context."
            )
        if parent_branch_id is None:
            output = self._recompute_all(hidden_states, attention_mask, **kwargs)
            self._store_activations(branch_id, output, hidden_states)
            return output
        if self.scheduler is not None and not self.scheduler.should_fold(self.layer_idx, step_idx):
            output = self._recompute_all(hidden_states, attention_mask, **kwargs)
            self._store_activations(branch_id, output, hidden_states)
            return output
        if self.scheduler is not None:
            self.gate.set_tau(self.scheduler.get_tau(layer_idx=self.layer_idx, step_idx=step_idx, task_type="general"))

        B, T = hidden_states.shape[:2]
        # Parent layer input (cache.get with an all-ones mask, folded_transformer.py:124-141).
        h_parent = None
        try:
            h_parent = self.cache.dense_rows(parent_branch_id, self.layer_idx, "hidden_states", T)
            if h_parent is not None:
                self.cache.touch(parent_branch_id, self.layer_idx, None, T)
                if h_parent.shape[0] == 1 and B > 1:
                    h_parent = h_parent.expand(B, *h_parent.shape[1:])
            else:
                ones = torch.ones((B, T), dtype=torch.bool, device=hidden_states.device)
                h_parent = _dense_get(self.cache, parent_branch_id, self.layer_idx, ones).get("hidden_states")
        except (KeyError, RuntimeError):
            h_parent = None
        if h_parent is None:
            output = self._recompute_all(hidden_states, attention_mask, **kwargs)
            self._store_activations(branch_id, output, hidden_states)
            return output
        h_parent = h_parent.to(dtype=hidden_states.dtype, device=hidden_states.device)

        g = self.gate.forward_compact(hidden_states, h_parent)
        stable_mask = g.stable_mask
        GLOBAL_STABILITY_PROFILER.record(
            branch_id=branch_id,
            parent_branch_id=parent_branch_id,
            layer_idx=self.layer_idx,
            step_idx=step_idx,
            stable_mask=stable_mask,
            tau=self.gate.tau,
            metric=self.gate.metric,
        )
        # The single host synchronisation of this layer: divergent total + per-token "any stable".
        host = torch.cat([g.div_count.sum().view(1), stable_mask.any(dim=0).to(torch.int32)]).cpu().numpy()
        n_div, any_stable = int(host[0]), host[1:].astype(bool)

        if n_div == 0:  # all stable -> parent output (folded_transformer.py:162-179)
            ffn_out = None
            try:
                ffn_out = _dense_get(self.cache, parent_branch_id, self.layer_idx, stable_mask).get("ffn_out")
            except (KeyError, RuntimeError):
                ffn_out = None
            if ffn_out is not None:
                self._store_activations(branch_id, ffn_out, hidden_states)
                return ffn_out
            output = self._recompute_all(hidden_states, attention_mask, **kwargs)
            self._store_activations(branch_id, output, hidden_states)
            return output
        if n_div == B * T:  # nothing stable -> recompute (folded_transformer.py:183-186)
            output = self._recompute_all(hidden_states, attention_mask, **kwargs)
            self._store_activations(branch_id, output, hidden_states)
            return output

        parent_ffn = self._get_parent_ffn_output(parent_branch_id, stable_mask, any_stable, T)
        child_out = self._recompute_all(hidden_states, attention_mask, **kwargs)
        if parent_ffn.shape[0] == 1 and B > 1:
            parent_ffn = parent_ffn.expand(B, *parent_ffn.shape[1:])
        h_out = merge_stable_divergent(parent_ffn, child_out, stable_mask)
        self._store_activations(branch_id, h_out, hidden_states)
        return h_out

    def _get_parent_ffn_output(self, parent_branch_id, stable_mask: torch.Tensor, any_stable: np.ndarray, T: int) -> torch.Tensor:
        """Parent ``ffn_out`` rows for the merge; RuntimeError when the parent has none."""
        rows = self.cache.dense_rows(parent_branch_id, self.layer_idx, "ffn_out", T)
        if rows is not None:
            self.cache.touch(parent_branch_id, self.layer_idx, any_stable, T)
            return rows
        acts = _dense_get(self.cache, parent_branch_id, self.layer_idx, stable_mask)
        ffn_out = acts.get("ffn_out")
        if ffn_out is None:
            raise RuntimeError(f"Parent FFN output missing for branch={parent_branch_id}, layer={self.layer_idx}")
        return ffn_out

    def _recompute_all(self, hidden_states: torch.Tensor, attention_mask: torch.Tensor | None, **kwargs: Any) -> torch.Tensor:
        """Run the wrapped layer on every row; the first element of a tuple output is the result."""
        sig = inspect.signature(self.original_layer.forward)
        accepted = set(sig.parameters)
        has_varkw = any(p.kind == inspect.Parameter.VAR_KEYWORD for p in sig.parameters.values())
        layer_kwargs = {k: v for k, v in kwargs.items() if k not in _ACTFOLD_KWARGS}
        if not has_varkw:
            layer_kwargs = {k: v for k, v in layer_kwargs.items() if k in accepted}
        if attention_mask is not None and "attention_mask" in accepted:
            layer_kwargs["attention_mask"] = attention_mask
        raw = self.original_layer(hidden_states, **layer_kwargs)
        return raw[0] if isinstance(raw, tuple) else raw

    def _store_activations(self, branch_id: str, ffn_out: torch.Tensor, hidden_states: torch.Tensor) -> None:
        self.cache.put(branch_id=branch_id, layer_idx=self.layer_idx, activations={"ffn_out": ffn_out, "hidden_states": hidden_states})
