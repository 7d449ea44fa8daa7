"""ActivationCache restated with per-token dict entries (TEST INFRASTRUCTURE).

Follows actfold/core/activation_cache.py:
  * put  :50-110  per-token entries keyed (branch, layer, token, step); LRU
                  eviction of the oldest entry once a layer holds more than
                  ``max_entries`` tokens (:109-110)
  * get  :112-153 zero-filled reconstruction through gather_cached_activations
                  (KeyError when token 0 is missing) and an LRU touch of every
                  token selected by any batch row (:147-151)
  * clear_branch / clear_layer / clear_all / num_entries :155-175

Pure Python: only for the small cases the tests use.
"""

from __future__ import annotations

from collections import OrderedDict

import numpy as np

from oracle.rows import gather_dense, gather_sparse


class OracleActivationCache:
    def __init__(self, max_entries_per_layer: int = 1024) -> None:
        self.max_entries = max_entries_per_layer
        self._caches: dict[int, OrderedDict] = {}

    def put(self, branch_id, layer_idx: int, activations: dict[str, np.ndarray], step_idx: int = 0) -> None:
        if not activations:
            raise ValueError("activations must not be empty")
        cache = self._caches.setdefault(layer_idx, OrderedDict())
        expected = None
        for name, t in activations.items():
            if t.ndim < 2:
                raise ValueError(f"Activation '{name}' must have at least 2 leading dimensions")
            if expected is None:
                expected = t.shape[:2]
            elif t.shape[:2] != expected:
                raise ValueError(f"Activation '{name}' has inconsistent leading shape")
        _, T = expected
        for tok in range(T):
            key = (branch_id, layer_idx, tok, step_idx)
            val = {n: np.array(a[:, tok]) for n, a in activations.items()}
            if key in cache:
                cache.move_to_end(key)
            cache[key] = val
            if len(cache) > self.max_entries:
                cache.popitem(last=False)

    def get(self, branch_id, layer_idx: int, token_mask: np.ndarray, step_idx: int = 0) -> dict[str, np.ndarray]:
        cache = self._caches.setdefault(layer_idx, OrderedDict())
        B, T = token_mask.shape
        k0 = (branch_id, layer_idx, 0, step_idx)
        if k0 not in cache:
            raise KeyError(f"No cache entry for branch={branch_id}, layer={layer_idx}, step={step_idx}")
        sample = cache[k0]
        dense = all((branch_id, layer_idx, t, step_idx) in cache for t in range(T))
        out: dict[str, np.ndarray] = {}
        for name, s in sample.items():
            if dense:
                stacked = np.stack([cache[(branch_id, layer_idx, t, step_idx)][name] for t in range(T)], axis=1)
                out[name] = gather_dense(stacked, token_mask)
            else:
                per_tok = {
                    t: cache[(branch_id, layer_idx, t, step_idx)][name]
                    for t in range(T)
                    if (branch_id, layer_idx, t, step_idx) in cache
                }
                out[name] = gather_sparse(per_tok, token_mask, s.shape[1:], s.dtype)
        for t in range(T):
            key = (branch_id, layer_idx, t, step_idx)
            if key in cache and token_mask[:, t].any():
                cache.move_to_end(key)
        return out

    def clear_branch(self, branch_id) -> None:
        for cache in self._caches.values():
            for key in [k for k in cache if k[0] == branch_id]:
                del cache[key]

    def clear_layer(self, layer_idx: int) -> None:
        if layer_idx in self._caches:
            self._caches[layer_idx].clear()

    def clear_all(self) -> None:
        self._caches.clear()

    def num_entries(self, layer_idx: int | None = None) -> int:
        if layer_idx is not None:
            return len(self._caches.get(layer_idx, {}))
        return sum(len(c) for c in self._caches.values())

    def present_tokens(self, branch_id, layer_idx: int, T: int, step_idx: int = 0) -> np.ndarray:
        cache = self._caches.get(layer_idx, {})
        return np.array([(branch_id, layer_idx, t, step_idx) in cache for t in range(T)])
