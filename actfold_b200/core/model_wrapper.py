"""FoldedModel: wrap a model so its layer stack verifies branches by folding.

Drop-in for actfold/core/model_wrapper.py:19-216: same layer-path discovery,
``forward(tokens, branch_id, parent_branch_id=None, attention_mask=None,
step_idx=0, **kwargs)``, kwargs fallback on TypeError, ``restore`` and
``folding_applied``.

Models that implement the native folded protocol (``actfold_b200.llada``
models expose ``native_folded_forward``) are routed to the batched CUDA pass,
which gates, packs and recomputes only divergent rows of all children at
once; every other model goes through FoldedTransformerLayer per layer.
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


class FoldedModel(nn.Module):
    _DEFAULT_LAYER_PATHS: tuple[str, ...] = (
        "model.layers",
        "transformer.h",
        "transformer.layers",
        "layers",
        "h",
        "gpt_neox.layers",
        "transformer.blocks",
        "blocks",
        "model.decoder.layers",
        "decoder.layers",
        "encoder.layer",
        "model.encoder.layer",
        "bert.encoder.layer",
        "decoder.block",
        "model.decoder.block",
        "encoder.block",
        "model.encoder.block",
    )

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
        self.layer_names = layer_names or self._DEFAULT_LAYER_PATHS
        self._layer_path: str | None = None
        self._original_layers: nn.ModuleList | None = None
        self._wrapped_layers: nn.ModuleList | None = None
        self._native = callable(getattr(model, "native_folded_forward", None))
        self._apply_folding()

    def _apply_folding(self) -> None:
        for path in self.layer_names:
            layer_list = self._get_attr_path(self.wrapped_model, path)
            if isinstance(layer_list, nn.ModuleList):
                self._layer_path = path
                self._original_layers = layer_list
                self._wrapped_layers = nn.ModuleList(
                    FoldedTransformerLayer(original_layer=layer, cache=self.cache, gate=self.gate, layer_idx=idx, scheduler=self.scheduler)
                    for idx, layer in enumerate(layer_list)
                )
                if not self._native:
                    self._set_attr_path(self.wrapped_model, path, self._wrapped_layers)
                return
        warnings.warn(
            "FoldedModel could not find a known layer stack in the base model. "
            f"Searched: {self.layer_names}. Folding is disabled and the wrapper acts as a thin pass-through.",
            stacklevel=2,
        )

    @staticmethod
    def _get_attr_path(obj: nn.Module, path: str) -> nn.ModuleList | None:
        current: Any = obj
        for part in path.split("."):
            if not hasattr(current, part):
                return None
            current = getattr(current, part)
        return current if isinstance(current, nn.ModuleList) else None

    @staticmethod
    def _set_attr_path(obj: nn.Module, path: str, value: nn.ModuleList) -> None:
        parts = path.split(".")
        current: Any = obj
        for part in parts[:-1]:
            current = getattr(current, part)
        setattr(current, parts[-1], value)

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
        actfold_keys = {"branch_id", "parent_branch_id", "step_idx"}
        if self._native and self.folding_applied:
            return self.wrapped_model.native_folded_forward(
                tokens,
                cache=self.cache,
                gate=self.gate,
                branch_id=branch_id,
                parent_branch_id=parent_branch_id,
                step_idx=step_idx,
                scheduler=self.scheduler,
                **kwargs,
            )
        if not self.folding_applied:
            forward_kwargs: dict[str, Any] = {k: v for k, v in kwargs.items() if k not in actfold_keys}
            if attention_mask is not None and "attention_mask" in inspect.signature(self.wrapped_model.forward).parameters:
                forward_kwargs["attention_mask"] = attention_mask
            return self.wrapped_model(tokens, **forward_kwargs)
        with folding_scope(branch_id, parent_branch_id, step_idx):
            forward_kwargs = {**kwargs, "branch_id": branch_id, "parent_branch_id": parent_branch_id, "step_idx": step_idx}
            sig = inspect.signature(self.wrapped_model.forward)
            if attention_mask is not None and "attention_mask" in sig.parameters:
                forward_kwargs["attention_mask"] = attention_mask
            try:
                out = self.wrapped_model(tokens, **forward_kwargs)
            except TypeError as exc:
                if any(key in str(exc) for key in actfold_keys):
                    fallback = {k: v for k, v in kwargs.items() if k not in actfold_keys}
                    if attention_mask is not None and "attention_mask" in sig.parameters:
                        fallback["attention_mask"] = attention_mask
                    out = self.wrapped_model(tokens, **fallback)
                else:
                    raise
        return out

    def restore(self) -> nn.Module:
        if self._layer_path is not None and self._original_layers is not None:
            if not self._native:
                self._set_attr_path(self.wrapped_model, self._layer_path, self._original_layers)
            self._wrapped_layers = None
        return self.wrapped_model
