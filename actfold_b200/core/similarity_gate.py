"""SimilarityGate on the CUDA gate kernel.

Drop-in for actfold/core/similarity_gate.py:10-112: same constructor,
validation messages, ``forward(h_child, h_parent) -> BoolTensor[B, T]`` and
``set_tau``. The similarity (cosine, l2 or pearson) and the threshold run in
``af_gate`` with the reference's rounding chain, so masks match the reference
bit for bit except for rows whose float32 similarity sits on the decision
boundary. ``forward_compact`` additionally returns the order-preserving
divergent index lists and counts computed in the same launch.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from actfold_b200 import _lib


class GateResult:
    """Mask plus fused compaction of one gate call (all on the device)."""

    __slots__ = ("stable_mask", "div_idx", "div_count", "stable_idx", "sim")

    def __init__(self, stable_mask, div_idx=None, div_count=None, stable_idx=None, sim=None):
        self.stable_mask = stable_mask
        self.div_idx = div_idx
        self.div_count = div_count
        self.stable_idx = stable_idx
        self.sim = sim


class SimilarityGate(nn.Module):
    """Boolean stability mask from parent/child hidden states (True = stable)."""

    def __init__(self, tau: float = 0.95, metric: str = "cosine", eps: float = 1e-8) -> None:
        super().__init__()
        if not 0.0 <= tau <= 1.0:
            raise ValueError(f"tau must be in [0, 1], got {tau}")
        if metric not in {"cosine", "l2", "pearson"}:
            raise ValueError(f"Unsupported metric: {metric}")
        self.tau = tau
        self.metric = metric
        self.eps = eps

    @staticmethod
    def _validate(h_child: torch.Tensor, h_parent: torch.Tensor) -> None:
        if h_child.ndim != 3 or h_parent.ndim != 3:
            raise ValueError(
                f"SimilarityGate expects 3-D inputs [B, T, H], got "
                f"h_child {h_child.shape} and h_parent {h_parent.shape}"
            )
        if h_child.shape != h_parent.shape:
            raise ValueError(f"Shape mismatch: h_child {h_child.shape} vs h_parent {h_parent.shape}")

    def _run(self, h_child: torch.Tensor, h_parent: torch.Tensor, compact: bool, want_sim: bool, want_stable_idx: bool) -> GateResult:
        self._validate(h_child, h_parent)
        _lib.require_cuda(h_child, what="SimilarityGate")
        if h_child.dtype not in _lib.DTYPE:
            raise ValueError(f"SimilarityGate: unsupported dtype {h_child.dtype}")
        # Align parent to the child's device/dtype (similarity_gate.py:70-71).
        h_parent = h_parent.to(dtype=h_child.dtype, device=h_child.device)
        B, T, H = h_child.shape
        if h_child.stride(2) != 1:
            h_child = h_child.contiguous()
        if h_parent.stride(2) != 1:
            h_parent = h_parent.contiguous()
        es = h_child.element_size()
        dev = h_child.device
        mask = torch.empty((B, T), dtype=torch.bool, device=dev)
        sim = torch.empty((B, T), dtype=torch.float32, device=dev) if want_sim else None
        div_idx = torch.empty((B, T), dtype=torch.int32, device=dev) if compact else None
        div_cnt = torch.empty((B,), dtype=torch.int32, device=dev) if compact else None
        st_idx = torch.empty((B, T), dtype=torch.int32, device=dev) if (compact and want_stable_idx) else None
        lib = _lib.load()
        with torch.cuda.device(dev):
            st = lib.af_gate(
                h_child.data_ptr(), h_child.stride(0) * es, h_child.stride(1) * es,
                h_parent.data_ptr(), h_parent.stride(0) * es, h_parent.stride(1) * es,
                B, T, H, _lib.DTYPE[h_child.dtype], _lib.METRIC[self.metric],
                float(self.tau), float(self.eps), float(H ** 0.5 + self.eps),
                mask.data_ptr(), T, _lib.ptr(sim), _lib.ptr(st_idx), _lib.ptr(div_idx), T, _lib.ptr(div_cnt),
                _lib.stream_ptr(dev),
            )
        _lib.check(st, "af_gate")
        return GateResult(mask, div_idx, div_cnt, st_idx, sim)

    def forward(self, h_child: torch.Tensor, h_parent: torch.Tensor) -> torch.Tensor:
        """Return the stability mask ``[B, T]`` (True = stable)."""
        return self._run(h_child, h_parent, compact=False, want_sim=False, want_stable_idx=False).stable_mask

    def forward_compact(self, h_child: torch.Tensor, h_parent: torch.Tensor, stable_idx: bool = False) -> GateResult:
        """Mask plus divergent index lists ``[B, T]`` (-1 padded) and counts ``[B]``."""
        return self._run(h_child, h_parent, compact=True, want_sim=False, want_stable_idx=stable_idx)

    def similarity(self, h_child: torch.Tensor, h_parent: torch.Tensor) -> torch.Tensor:
        """Per-token similarity (float32 holding the value rounded to the input dtype)."""
        return self._run(h_child, h_parent, compact=False, want_sim=True, want_stable_idx=False).sim

    def _compute_similarity(self, h_child: torch.Tensor, h_parent: torch.Tensor) -> torch.Tensor:
        return self.similarity(h_child, h_parent).to(h_child.dtype)

    def set_tau(self, tau: float) -> None:
        if not 0.0 <= tau <= 1.0:
            raise ValueError(f"tau must be in [0, 1], got {tau}")
        self.tau = tau

    def extra_repr(self) -> str:
        return f"tau={self.tau}, metric={self.metric}, eps={self.eps}"
