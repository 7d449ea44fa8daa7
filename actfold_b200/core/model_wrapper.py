"""FoldedModel: a model whose layer stack verifies child branches by folding.

Public surface of actfold/core/model_wrapper.py:19-216 (constructor
arguments, ``forward(tokens, branch_id, parent_branch_id=None,
attention_mask=None, step_idx=0, **kwargs)``, ``restore()``,
``folding_applied``, the searched layer paths and their order, the warning
when no stack is found, the retry without branch arguments when the base
model rejects them).

Two ways to run a child, chosen once at construction:

* native -- the wrapped model implements ``native_folded_forward`` (the
  LLaDA / Dream models of ``actfold_b200.llada``): the whole batch of children
  runs as one CUDA pass that gates, packs and recomputes only divergent rows.
  The model's own layers are left in place.
* generic -- any other ``nn.Module`` with a discoverable layer stack: the
  stack is swapped for FoldedTransformerLayer wrappers and the model's own
  forward runs under the branch context.
"""

from __future__ import annotations

import inspect
import warnings
from typing import Any

import torch
import torch.nn as nn

from actfold_b200.core.folded_transformer import FoldedTransformerLayer
from actfold_b200.core.folding_context import folding_scope
from actfold_b200.core.folding_scheduler import FoldingScheduler
from actfold_b200.core.similarity_gate import SimilarityGate

# Where model families keep their block list, searched in this order (the
# reference's table; the first ModuleList found is the one wrapped).
LAYER_PATHS: tuple[str, ...] = (
    "model.layers", "transformer.h", "transformer.layers", "layers", "h",
    "gpt_neox.layers", "transformer.blocks", "blocks",
    "model.decoder.layers", "decoder.layers",
    "encoder.layer", "model.encoder.layer", "bert.encoder.layer",
    "decoder.block", "model.decoder.block", "encoder.block", "model.encoder.block",
)

_BRANCH_KEYS = ("branch_id", "parent_branch_id", "step_idx")


def locate_stack(model: nn.Module, paths) -> tuple[str, Any, str, nn.ModuleList] | None:
    """First ``path`` that names an nn.ModuleList: (path, owning object, attribute name, the list)."""
    for path in paths:
        *heads, last = path.split(".")
        owner: Any = model
        for name in heads:
            owner = getattr(owner, name, None)
            if owner is None:
                break
        stack = getattr(owner, last, None) if owner is not None else None
        if isinstance(stack, nn.ModuleList):
            return path, owner, last, stack
    return None


def _accepts(fn, name: str) -> bool:
    try:
        return name in inspect.signature(fn).parameters
    except (TypeError, ValueError):
        return False


class FoldedModel(nn.Module):
    _DEFAULT_LAYER_PATHS = LAYER_PATHS

    def __init__(
        self,
        model: nn.Module,
        cache,
        gate: SimilarityGate,
        layer_names: tuple[str, ...] | None = None,
        scheduler: FoldingScheduler | None = None,
    ) -> None:
        super().__init__()
        self.wrapped_model = model
        self.cache = cache
        self.gate = gate
        self.scheduler = scheduler
        self.layer_names = layer_names or LAYER_PATHS
        self._native = callable(getattr(model, "native_folded_forward", None))
        self._layer_path: str | None = None
        self._slot: tuple[Any, str] | None = None      # (owner, attribute) of the wrapped stack
        self._original_layers: nn.ModuleList | None = None
        self._wrapped_layers: nn.ModuleList | None = None
        found = locate_stack(model, self.layer_names)
        if found is None:
            warnings.warn(
                "FoldedModel could not find a known layer stack in the base model. "
                f"Searched: {self.layer_names}. Folding is disabled and the wrapper acts as a thin pass-through.",
                stacklevel=2,
            )
            return
        self._layer_path, owner, attr, stack = found
        self._slot = (owner, attr)
        self._original_layers = stack
        self._wrapped_layers = nn.ModuleList(
            FoldedTransformerLayer(original_layer=blk, cache=cache, gate=gate, layer_idx=i, scheduler=scheduler)
            for i, blk in enumerate(stack))
        if not self._native:  # the native pass reads the model's own weights; nothing is swapped
            setattr(owner, attr, self._wrapped_layers)

    @property
    def folding_applied(self) -> bool:
        return self._wrapped_layers is not None

    def forward(
        self,
        tokens: torch.Tensor,
        branch_id: str,
        parent_branch_id: str | None = None,
        attention_mask: torch.Tensor | None = None,
        step_idx: int = 0,
        **kwargs: Any,
    ) -> torch.Tensor:
        if self._native and self.folding_applied:
            return self.wrapped_model.native_folded_forward(
                tokens, cache=self.cache, gate=self.gate, branch_id=branch_id, parent_branch_id=parent_branch_id,
                step_idx=step_idx, scheduler=self.scheduler, **kwargs)
        plain = {k: v for k, v in kwargs.items() if k not in _BRANCH_KEYS}
        if attention_mask is not None and _accepts(self.wrapped_model.forward, "attention_mask"):
            plain["attention_mask"] = attention_mask
        if not self.folding_applied:
            return self.wrapped_model(tokens, **plain)
        branch = {"branch_id": branch_id, "parent_branch_id": parent_branch_id, "step_idx": step_idx}
        with folding_scope(branch_id, parent_branch_id, step_idx):
            try:
                return self.wrapped_model(tokens, **{**kwargs, **plain, **branch})
            except TypeError as exc:
                # A base model that rejects the branch arguments still folds:
                # its layers read them from the folding context instead.
                if not any(k in str(exc) for k in _BRANCH_KEYS):
                    raise
                return self.wrapped_model(tokens, **plain)

    def restore(self) -> nn.Module:
        if self._slot is not None and self._original_layers is not None:
            if not self._native:
                setattr(*self._slot, self._original_layers)
            self._wrapped_layers = None
        return self.wrapped_model
