"""Per-layer / per-step threshold schedule (host-side arithmetic only).

Same decisions as actfold/core/folding_scheduler.py:6-115:
``get_tau`` = base + layer bias (early layers +) + step bias (early steps -)
+ task bias, clamped to [0.80, 0.99]; ``should_fold`` is False for disabled
layers, the final layer and the final step.
"""

from __future__ import annotations


class FoldingScheduler:
    def __init__(
        self,
        base_tau: float = 0.95,
        num_layers: int = 12,
        num_steps: int = 10,
        disabled_layers: set[int] | None = None,
    ) -> None:
        if not 0.0 <= base_tau <= 1.0:
            raise ValueError(f"base_tau must be in [0, 1], got {base_tau}")
        if num_layers <= 0 or num_steps <= 0:
            raise ValueError("num_layers and num_steps must be positive.")
        self.base_tau = base_tau
        self.num_layers = num_layers
        self.num_steps = num_steps
        self.disabled_layers = set(disabled_layers or [])
        self.layer_bias_scale = 0.03
        self.step_bias_scale = 0.04
        self.task_bias: dict[str, float] = {"math": -0.03, "code": 0.03, "general": 0.0}

    def get_tau(self, layer_idx: int, step_idx: int, task_type: str = "general") -> float:
        if not 0 <= layer_idx < self.num_layers:
            raise ValueError(f"layer_idx {layer_idx} out of range [0, {self.num_layers})")
        if not 0 <= step_idx < self.num_steps:
            raise ValueError(f"step_idx {step_idx} out of range [0, {self.num_steps})")
        depth = 1.0 - layer_idx / max(self.num_layers - 1, 1)
        step = 1.0 - step_idx / max(self.num_steps - 1, 1)
        tau = (
            self.base_tau
            + self.layer_bias_scale * (2.0 * depth - 1.0)
            - self.step_bias_scale * step
            + self.task_bias.get(task_type, 0.0)
        )
        return float(min(max(tau, 0.80), 0.99))

    def disable_layers(self, layer_indices) -> None:
        self.disabled_layers.update(layer_indices)

    def enable_layers(self, layer_indices) -> None:
        self.disabled_layers.difference_update(layer_indices)

    def should_fold(self, layer_idx: int, step_idx: int) -> bool:
        if not 0 <= layer_idx < self.num_layers or not 0 <= step_idx < self.num_steps:
            return False
        if layer_idx in self.disabled_layers:
            return False
        return not (layer_idx == self.num_layers - 1 or step_idx == self.num_steps - 1)

    def set_task_bias(self, task_type: str, bias: float) -> None:
        self.task_bias[task_type] = bias
