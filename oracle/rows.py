"""Row merge / gather restated in numpy (TEST INFRASTRUCTURE).

Follows actfold/core/fused_ops.py:
  * _merge_stable_divergent_torch :38-51 and merge_stable_divergent :206-253
  * _gather_cached_activations_torch :54-87 (sparse path) and
    gather_cached_activations :256-324 (dense path)
"""

from __future__ import annotations

import numpy as np


def merge(parent: np.ndarray, child: np.ndarray, stable: np.ndarray) -> np.ndarray:
    """out[b, t] = parent[b, t] if stable[b, t] else child[b, t] (fused_ops.py:50-51)."""
    if parent.ndim != 3 or child.ndim != 3:
        raise ValueError("parent_ffn and child_out must be 3-D [B, T, H]")
    if parent.shape != child.shape:
        raise ValueError("Shape mismatch")
    if stable.ndim != 2 or stable.shape != parent.shape[:2]:
        raise ValueError("stable_mask must be 2-D [B, T]")
    return np.where(stable[..., None].astype(bool), parent, child)


def gather_dense(stacked: np.ndarray, token_mask: np.ndarray) -> np.ndarray:
    """Dense path (fused_ops.py:315-322): per-(b, t) zero-fill of a complete [B, T, ...] stack.

    A stored batch of 1 is broadcast to the requested batch (fused_ops.py:323-330).
    """
    B, T = token_mask.shape
    if stacked.shape[0] != B:
        stacked = np.broadcast_to(stacked, (B,) + stacked.shape[1:]) if stacked.shape[0] == 1 else stacked[:B]
    m = token_mask.reshape(B, T, *([1] * (stacked.ndim - 2))).astype(bool)
    return np.where(m, stacked, np.zeros_like(stacked))


def gather_sparse(per_token: dict[int, np.ndarray], token_mask: np.ndarray, trailing: tuple, dtype) -> np.ndarray:
    """Sparse path (fused_ops.py:74-87): a token is copied for every batch row when
    it is present and selected by ANY batch row; missing tokens stay zero."""
    B, T = token_mask.shape
    out = np.zeros((B, T) + tuple(trailing), dtype=dtype)
    for t in range(T):
        if t not in per_token:
            continue
        if not token_mask[:, t].any():
            continue
        out[:, t] = per_token[t]
    return out
