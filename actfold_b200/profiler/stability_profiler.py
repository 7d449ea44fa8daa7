"""Layer-aware stability profiler without per-layer host synchronisation.

Drop-in for actfold/profiler/stability_profiler.py:19-193 (same dataclasses,
``record`` / ``get_profile`` / ``get_mean_stable_ratio`` / ``reset*`` /
``set_enabled`` and the global instance). The reference's ``record`` calls
``.item()`` and ``nonzero`` on every layer, stalling the GPU each time. Here
``record`` only queues the device mask; pending records are resolved with
ONE device-to-host copy the first time statistics are read
(``get_profile``, ``get_mean_stable_ratio``, ``flush``). The native batched
pass feeds whole-pass device counters through ``record_batch``.
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field
from typing import Any, Optional, Sequence

import torch


@dataclass
class LayerStabilityStats:
    layer_idx: int
    step_idx: int
    stable_ratio: float
    tau_used: float
    metric: str
    num_tokens: int
    divergence_positions: Optional[torch.Tensor] = None

    def to_dict(self) -> dict[str, Any]:
        return {
            "layer_idx": self.layer_idx,
            "step_idx": self.step_idx,
            "stable_ratio": self.stable_ratio,
            "tau_used": self.tau_used,
            "metric": self.metric,
            "num_tokens": self.num_tokens,
            "divergence_positions": self.divergence_positions.tolist() if self.divergence_positions is not None else None,
        }


@dataclass
class StabilityProfile:
    branch_id: Any
    parent_branch_id: Optional[Any]
    layer_stats: list[LayerStabilityStats] = field(default_factory=list)

    @property
    def mean_stable_ratio(self) -> float:
        if not self.layer_stats:
            return 0.0
        return sum(s.stable_ratio for s in self.layer_stats) / len(self.layer_stats)

    @property
    def final_stable_ratio(self) -> float:
        return self.layer_stats[-1].stable_ratio if self.layer_stats else 0.0

    @property
    def min_stable_ratio(self) -> float:
        return min(s.stable_ratio for s in self.layer_stats) if self.layer_stats else 0.0

    def to_dict(self) -> dict[str, Any]:
        return {
            "branch_id": self.branch_id,
            "parent_branch_id": self.parent_branch_id,
            "mean_stable_ratio": self.mean_stable_ratio,
            "final_stable_ratio": self.final_stable_ratio,
            "min_stable_ratio": self.min_stable_ratio,
            "layer_stats": [s.to_dict() for s in self.layer_stats],
        }


class StabilityProfiler:
    def __init__(self, enabled: bool = True) -> None:
        self.enabled = enabled
        self._profiles: dict[Any, StabilityProfile] = {}
        self._history: dict[tuple[int, int], list[float]] = defaultdict(list)
        self._max_history_len = 100
        self._pending: list[tuple] = []

    def record(
        self,
        branch_id: Any,
        parent_branch_id: Optional[Any],
        layer_idx: int,
        step_idx: int,
        stable_mask: torch.Tensor,
        tau: float,
        metric: str = "cosine",
    ) -> None:
        """Queue one layer's stability decision (``stable_mask`` [B, T], True = stable)."""
        if not self.enabled:
            return
        self._pending.append(("mask", branch_id, parent_branch_id, layer_idx, step_idx, stable_mask.detach(), tau, metric))

    def record_batch(
        self,
        branch_ids: list[Any],
        parent_branch_id: Optional[Any],
        step_idx: int,
        masks: torch.Tensor,
        tau: float | Sequence[float],
        metric: str = "cosine",
        layer_offset: int = 0,
        layer_ids: Optional[Sequence[int]] = None,
    ) -> None:
        """Queue a whole pass: ``masks`` [n, C, T] (True = stable) for children ``branch_ids``.

        Row i of ``masks`` is layer ``layer_ids[i]`` (default ``layer_offset + i``);
        ``tau`` is one threshold for every row or one per row.
        """
        if not self.enabled:
            return
        layers = list(layer_ids) if layer_ids is not None else [layer_offset + i for i in range(masks.shape[0])]
        taus = list(tau) if isinstance(tau, (list, tuple)) else [tau] * len(layers)
        if len(layers) != masks.shape[0] or len(taus) != masks.shape[0]:
            raise ValueError("record_batch: one layer index and one tau per mask row")
        self._pending.append(("batch", list(branch_ids), parent_branch_id, layers, step_idx, masks.detach(), taus, metric))

    def flush(self) -> None:
        """Resolve queued records with one device-to-host copy."""
        if not self._pending:
            return
        pending, self._pending = self._pending, []
        host = [p[5].to("cpu", non_blocking=False) for p in pending] if pending else []
        for p, m in zip(pending, host):
            kind, bid, pid, layer, step, _, tau, metric = p
            if kind == "mask":
                self._add(bid, pid, layer, step, m.bool(), tau, metric)
            else:
                for li in range(m.shape[0]):
                    for ci, b in enumerate(bid):
                        self._add(b, pid, layer[li], step, m[li, ci][None].bool(), tau[li], metric)

    def _add(self, branch_id, parent_branch_id, layer_idx, step_idx, mask: torch.Tensor, tau, metric) -> None:
        num = int(mask.numel())
        ratio = float(mask.float().mean().item()) if num else 0.0
        div = torch.nonzero(~mask, as_tuple=False) if ratio < 1.0 else None
        stats = LayerStabilityStats(layer_idx, step_idx, ratio, tau, metric, num, div)
        if branch_id not in self._profiles:
            self._profiles[branch_id] = StabilityProfile(branch_id=branch_id, parent_branch_id=parent_branch_id)
        self._profiles[branch_id].layer_stats.append(stats)
        hist = self._history[(layer_idx, step_idx)]
        hist.append(ratio)
        if len(hist) > self._max_history_len:
            hist.pop(0)

    def get_profile(self, branch_id: Any) -> Optional[StabilityProfile]:
        self.flush()
        return self._profiles.get(branch_id)

    def get_mean_stable_ratio(self, layer_idx: int, step_idx: int = 0) -> Optional[float]:
        self.flush()
        hist = self._history.get((layer_idx, step_idx))
        if not hist:
            return None
        return sum(hist) / len(hist)

    def reset_branch(self, branch_id: Any) -> None:
        self.flush()
        self._profiles.pop(branch_id, None)

    def reset(self) -> None:
        self._pending.clear()
        self._profiles.clear()
        self._history.clear()

    def set_enabled(self, enabled: bool) -> None:
        self.enabled = enabled
        if not enabled:
            self.reset()


GLOBAL_STABILITY_PROFILER = StabilityProfiler(enabled=True)
