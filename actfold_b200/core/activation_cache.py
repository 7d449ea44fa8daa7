"""ActivationCache backed by dense device blocks.

Drop-in for actfold/core/activation_cache.py:12-175. The reference keeps one
dict entry per token, ``(branch, layer, token, step) -> {name: Tensor[B, ...]}``,
and rebuilds ``[B, T, ...]`` tensors with a Python loop and ``torch.stack``
on every ``get``. Here one ``put`` stores each activation as ONE contiguous
``[B, T, ...]`` device copy (a *block*), and ``get`` is a single
``af_gather_rows_masked`` launch per activation.

The reference's per-token LRU is kept exactly, without per-token Python
objects: each block carries a host array of per-token LRU stamps (-1 =
evicted). ``put`` stamps its tokens in order, ``get`` re-stamps every token
selected by any batch row, and when a layer holds more than
``max_entries_per_layer`` tokens the oldest stamps are evicted — the same
entries the reference's ``OrderedDict.popitem(last=False)`` loop removes.
Errors match the reference: ValueError for empty / inconsistent ``put``,
KeyError when token 0 of the requested (branch, layer, step) is missing.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

from actfold_b200 import _lib
from actfold_b200.core.fused_ops import masked_rows


class _Block:
    __slots__ = ("tensors", "stamps", "B", "T")

    def __init__(self, tensors: dict[str, torch.Tensor], B: int, T: int) -> None:
        self.tensors = tensors
        self.B = B
        self.T = T
        self.stamps = np.full(T, -1, dtype=np.int64)

    def present(self, T: int) -> np.ndarray:
        p = np.zeros(T, dtype=bool)
        n = min(T, self.T)
        p[:n] = self.stamps[:n] >= 0
        return p


def _validate_activations(activations: dict[str, torch.Tensor]) -> tuple[int, int]:
    if not activations:
        raise ValueError("activations must not be empty")
    expected = None
    for name, tensor in activations.items():
        if tensor.ndim < 2:
            raise ValueError(
                f"Activation '{name}' must have at least 2 leading dimensions [batch, seq_len, ...], got shape {tensor.shape}"
            )
        leading = tensor.shape[:2]
        if expected is None:
            expected = leading
        elif leading != expected:
            raise ValueError(f"Activation '{name}' has inconsistent leading shape {leading}; expected {expected}")
    return int(expected[0]), int(expected[1])


class ActivationCache:
    """Per-layer LRU cache of branch activations (token-granular accounting)."""

    def __init__(self, max_entries_per_layer: int = 1024, device: str = "cuda") -> None:
        self.max_entries = max_entries_per_layer
        self.device = device
        self._caches: dict[int, dict[tuple[Any, int], _Block]] = {}
        self._clock: dict[int, int] = {}

    # ------------------------------------------------------------------ helpers
    def _layer(self, layer_idx: int) -> dict[tuple[Any, int], _Block]:
        if layer_idx not in self._caches:
            self._caches[layer_idx] = {}
            self._clock[layer_idx] = 0
        return self._caches[layer_idx]

    def _stamp(self, layer_idx: int, blk: _Block, tokens: np.ndarray) -> None:
        """Give ``tokens`` (in order) the newest LRU stamps of the layer."""
        n = int(tokens.size)
        if n == 0:
            return
        c = self._clock[layer_idx]
        blk.stamps[tokens] = np.arange(c, c + n, dtype=np.int64)
        self._clock[layer_idx] = c + n

    def _evict(self, layer_idx: int) -> None:
        layer = self._caches[layer_idx]
        total = sum(int((b.stamps >= 0).sum()) for b in layer.values())
        excess = total - self.max_entries
        if excess <= 0:
            return
        keys = list(layer)
        stamps = np.concatenate([layer[k].stamps for k in keys])
        owner = np.concatenate([np.full(layer[k].T, i, dtype=np.int64) for i, k in enumerate(keys)])
        offs = np.concatenate([np.arange(layer[k].T) for k in keys])
        live = np.nonzero(stamps >= 0)[0]
        oldest = live[np.argsort(stamps[live], kind="stable")[:excess]]
        for j in oldest:
            layer[keys[owner[j]]].stamps[offs[j]] = -1
        for k in keys:
            if not (layer[k].stamps >= 0).any():
                del layer[k]

    def _block(self, branch_id: Any, layer_idx: int, step_idx: int) -> _Block | None:
        return self._caches.get(layer_idx, {}).get((branch_id, step_idx))

    def _touch(self, branch_id: Any, layer_idx: int, step_idx: int, selected: np.ndarray | None, T: int) -> None:
        """LRU touch of present tokens in [0, T) that are selected (None = all)."""
        blk = self._block(branch_id, layer_idx, step_idx)
        if blk is None:
            return
        pres = blk.present(T)
        if selected is not None:
            pres &= np.asarray(selected, dtype=bool)[:T]
        self._stamp(layer_idx, blk, np.nonzero(pres)[0])

    # ----------------------------------------------------------------- public
    def put(self, branch_id: Any, layer_idx: int, activations: dict[str, torch.Tensor], step_idx: int = 0) -> None:
        """Store ``[batch, seq_len, ...]`` activations for (branch, layer, step)."""
        B, T = _validate_activations(activations)
        _lib.require_cuda(*activations.values(), what="ActivationCache.put")
        layer = self._layer(layer_idx)
        key = (branch_id, step_idx)
        old = layer.get(key)
        tensors = {n: t.detach().contiguous().clone() if t.is_contiguous() else t.detach().contiguous() for n, t in activations.items()}
        if old is not None and old.T > T and old.B == B and set(old.tensors) == set(tensors) and all(
            old.tensors[n].shape[2:] == tensors[n].shape[2:] and old.tensors[n].dtype == tensors[n].dtype for n in tensors
        ):
            # A shorter re-put replaces tokens [0, T) and keeps the older tail entries.
            for n, t in tensors.items():
                old.tensors[n][:, :T].copy_(t)
            blk = old
        else:
            blk = _Block(tensors, B, T)
            layer[key] = blk
        self._stamp(layer_idx, blk, np.arange(T))
        self._evict(layer_idx)

    def put_views(self, branch_id: Any, layer_idx: int, activations: dict[str, torch.Tensor], step_idx: int = 0) -> None:
        """``put`` without copying: the cache keeps the given tensors (callers must not modify them).

        Used for the native parent pass, whose per-layer activations already
        live in one dense device buffer.
        """
        B, T = _validate_activations(activations)
        _lib.require_cuda(*activations.values(), what="ActivationCache.put_views")
        layer = self._layer(layer_idx)
        blk = _Block({n: t.detach() for n, t in activations.items()}, B, T)
        layer[(branch_id, step_idx)] = blk
        self._stamp(layer_idx, blk, np.arange(T))
        self._evict(layer_idx)

    def get(self, branch_id: Any, layer_idx: int, token_mask: torch.Tensor, step_idx: int = 0) -> dict[str, torch.Tensor]:
        """Zero-filled ``[B, T, ...]`` activations for tokens selected by ``token_mask``."""
        self._layer(layer_idx)
        blk = self._block(branch_id, layer_idx, step_idx)
        if blk is None or blk.stamps[0] < 0:
            raise KeyError(f"No cache entry for branch={branch_id}, layer={layer_idx}, step={step_idx}")
        B, T = token_mask.shape
        present = blk.present(T)
        dense = bool(present.all())
        out: dict[str, torch.Tensor] = {}
        for name, src in blk.tensors.items():
            _lib.require_cuda(src, what="ActivationCache.get")
            if T > blk.T:
                pad = torch.zeros((src.shape[0], T) + tuple(src.shape[2:]), dtype=src.dtype, device=src.device)
                pad[:, : blk.T].copy_(src)
                src = pad
            pres_t = None if dense else torch.from_numpy(present)
            out[name] = masked_rows(src[:, :T], token_mask, pres_t, dense)
        sel = token_mask.any(dim=0)
        self._touch(branch_id, layer_idx, step_idx, sel.cpu().numpy(), T)
        return out

    def clear_branch(self, branch_id: Any) -> None:
        """Evict all entries belonging to ``branch_id``."""
        for layer in self._caches.values():
            for key in [k for k in layer if k[0] == branch_id]:
                del layer[key]
        drop_native_branches(self, branch_id)

    def clear_layer(self, layer_idx: int) -> None:
        if layer_idx in self._caches:
            self._caches[layer_idx].clear()

    def clear_all(self) -> None:
        self._caches.clear()
        self._clock.clear()
        drop_native_branches(self)

    def num_entries(self, layer_idx: int | None = None) -> int:
        """Number of cached token entries, optionally for one layer."""
        layers = [self._caches.get(layer_idx, {})] if layer_idx is not None else list(self._caches.values())
        return int(sum(int((b.stamps >= 0).sum()) for layer in layers for b in layer.values()))

    # ----------------------------------------------------- folded-layer access
    def dense_rows(self, branch_id: Any, layer_idx: int, name: str, T: int, step_idx: int = 0) -> torch.Tensor | None:
        """The stored ``[Bs, T, ...]`` block of ``name`` when every token in [0, T) is cached, else None.

        No copy and no LRU touch; the folded layer uses this to feed the gate
        and the merge straight from the cache.
        """
        blk = self._block(branch_id, layer_idx, step_idx)
        if blk is None or name not in blk.tensors or T > blk.T or not blk.present(T).all():
            return None
        return blk.tensors[name][:, :T]

    def has_entry(self, branch_id: Any, layer_idx: int, step_idx: int = 0) -> bool:
        blk = self._block(branch_id, layer_idx, step_idx)
        return blk is not None and blk.stamps[0] >= 0

    def touch(self, branch_id: Any, layer_idx: int, selected: np.ndarray | None, T: int, step_idx: int = 0) -> None:
        """Apply the LRU touch of a ``get`` whose mask selects ``selected`` tokens (None = all)."""
        self._touch(branch_id, layer_idx, step_idx, selected, T)


def drop_native_branches(cache: Any, branch_id: Any = None) -> None:
    """Forget the native pass's dense parent caches and promotable children (all, or one branch)."""
    for attr in ("native_parents", "native_children"):
        d = getattr(cache, attr, None)
        if d is None:
            continue
        if branch_id is None:
            d.clear()
        else:
            d.pop(branch_id, None)
