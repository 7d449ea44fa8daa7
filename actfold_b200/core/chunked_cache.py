"""ChunkedActivationCache backed by dense device blocks.

Drop-in for actfold/core/chunked_cache.py:28-265: activations are accounted
in chunks of ``chunk_size`` tokens with an LRU over chunks
(``max_chunks = max(1, max_entries_per_layer // chunk_size)``), ``get``
returns the GATHERED subset ``[B, n_selected, ...]`` of tokens selected by any
batch row (missing chunks read as zero) or ``{}`` when no chunk of the
branch is cached, and ``num_entries`` counts chunks.

Storage is one contiguous ``[B, T, ...]`` device copy per put; chunk presence
and LRU order are host arrays. ``get`` is one ``af_gather_rows_index`` launch
per activation.

Deviation, on purpose: the reference FoldedTransformerLayer merges the
subset-shaped ``get`` result with a full-shape child output, which raises
"Shape mismatch" for any partially stable layer. The folded layer here reads
chunked caches through :meth:`get_dense` (zero-filled full shape, the
ActivationCache contract), so chunked caches fold correctly; ``get`` itself
keeps the reference's subset semantics.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

from actfold_b200 import _lib
from actfold_b200.core.activation_cache import _validate_activations, drop_native_branches
from actfold_b200.core.fused_ops import masked_rows


class _ChunkBlock:
    __slots__ = ("tensors", "stamps", "B", "T", "chunk")

    def __init__(self, tensors: dict[str, torch.Tensor], B: int, T: int, chunk: int) -> None:
        self.tensors = tensors
        self.B, self.T, self.chunk = B, T, chunk
        self.stamps = np.full((T + chunk - 1) // chunk, -1, dtype=np.int64)

    def token_present(self, T: int) -> np.ndarray:
        p = np.zeros(T, dtype=bool)
        n = min(T, self.T)
        chunk_live = self.stamps >= 0
        p[:n] = np.repeat(chunk_live, self.chunk)[:n]
        return p


class ChunkedActivationCache:
    def __init__(self, max_entries_per_layer: int = 1024, chunk_size: int = 64, device: str = "cuda") -> None:
        if chunk_size <= 0:
            raise ValueError(f"chunk_size must be positive, got {chunk_size}")
        if max_entries_per_layer <= 0:
            raise ValueError(f"max_entries_per_layer must be positive, got {max_entries_per_layer}")
        self.chunk_size = chunk_size
        self.max_entries = max_entries_per_layer
        self.max_chunks = max(1, max_entries_per_layer // chunk_size)
        self.device = device
        self._caches: dict[int, dict[tuple[Any, int], _ChunkBlock]] = {}
        self._clock: dict[int, int] = {}

    def _layer(self, layer_idx: int) -> dict[tuple[Any, int], _ChunkBlock]:
        if layer_idx not in self._caches:
            self._caches[layer_idx] = {}
            self._clock[layer_idx] = 0
        return self._caches[layer_idx]

    def _stamp(self, layer_idx: int, blk: _ChunkBlock, chunks: np.ndarray) -> None:
        n = int(chunks.size)
        if n:
            c = self._clock[layer_idx]
            blk.stamps[chunks] = np.arange(c, c + n, dtype=np.int64)
            self._clock[layer_idx] = c + n

    def _evict(self, layer_idx: int) -> None:
        layer = self._caches[layer_idx]
        keys = list(layer)
        total = sum(int((layer[k].stamps >= 0).sum()) for k in keys)
        excess = total - self.max_chunks
        if excess <= 0:
            return
        stamps = np.concatenate([layer[k].stamps for k in keys])
        owner = np.concatenate([np.full(layer[k].stamps.size, i) for i, k in enumerate(keys)])
        offs = np.concatenate([np.arange(layer[k].stamps.size) for k in keys])
        live = np.nonzero(stamps >= 0)[0]
        for j in live[np.argsort(stamps[live], kind="stable")[:excess]]:
            layer[keys[owner[j]]].stamps[offs[j]] = -1
        for k in keys:
            if not (layer[k].stamps >= 0).any():
                del layer[k]

    def put(self, branch_id: Any, layer_idx: int, activations: dict[str, torch.Tensor], step_idx: int = 0) -> None:
        B, T = _validate_activations(activations)
        _lib.require_cuda(*activations.values(), what="ChunkedActivationCache.put")
        layer = self._layer(layer_idx)
        tensors = {n: t.detach().contiguous().clone() for n, t in activations.items()}
        blk = _ChunkBlock(tensors, B, T, self.chunk_size)
        layer[(branch_id, step_idx)] = blk
        self._stamp(layer_idx, blk, np.arange(blk.stamps.size))
        self._evict(layer_idx)

    def _lookup(self, branch_id: Any, layer_idx: int, step_idx: int, T: int) -> _ChunkBlock | None:
        self._layer(layer_idx)
        blk = self._caches[layer_idx].get((branch_id, step_idx))
        if blk is None:
            return None
        n_chunks = (T + self.chunk_size - 1) // self.chunk_size
        live = np.nonzero(blk.stamps[:n_chunks] >= 0)[0]
        if live.size == 0:
            return None
        self._stamp(layer_idx, blk, live)  # touch, in chunk order
        return blk

    def get(self, branch_id: Any, layer_idx: int, token_mask: torch.Tensor, step_idx: int = 0) -> dict[str, torch.Tensor]:
        """Gathered ``[B, n_selected, ...]`` activations of tokens selected by any batch row."""
        B, T = token_mask.shape
        blk = self._lookup(branch_id, layer_idx, step_idx, T)
        if blk is None:
            return {}
        present = blk.token_present(T)
        sel = np.nonzero(token_mask.any(dim=0).cpu().numpy())[0]
        idx = np.where(present[sel], sel, -1).astype(np.int32)
        out: dict[str, torch.Tensor] = {}
        for name, src in blk.tensors.items():
            dev = src.device
            Bs = src.shape[0]
            if Bs != B and Bs != 1:
                raise RuntimeError(f"cached batch {Bs} cannot be broadcast to requested batch {B}")
            trailing = tuple(src.shape[2:])
            res = torch.empty((B, idx.size) + trailing, dtype=src.dtype, device=dev)
            if idx.size:
                idx_t = torch.from_numpy(idx).to(dev)
                es = src.element_size()
                row = int(np.prod(trailing)) if trailing else 1
                with torch.cuda.device(dev):
                    st = _lib.load().af_gather_rows_index(
                        src.data_ptr(), 0 if Bs == 1 else src.stride(0) * es, src.stride(1) * es,
                        idx_t.data_ptr(), idx.size, B, res.data_ptr(), res.stride(0) * es, res.stride(1) * es,
                        row * es, _lib.stream_ptr(dev),
                    )
                _lib.check(st, "ChunkedActivationCache.get")
            out[name] = res
        return out

    def get_dense(self, branch_id: Any, layer_idx: int, token_mask: torch.Tensor, step_idx: int = 0) -> dict[str, torch.Tensor]:
        """Zero-filled ``[B, T, ...]`` activations (ActivationCache.get contract); KeyError if nothing cached."""
        B, T = token_mask.shape
        blk = self._lookup(branch_id, layer_idx, step_idx, T)
        if blk is None:
            raise KeyError(f"No cache entry for branch={branch_id}, layer={layer_idx}, step={step_idx}")
        present = blk.token_present(T)
        dense = bool(present.all())
        out = {}
        for name, src in blk.tensors.items():
            if T > blk.T:
                pad = torch.zeros((src.shape[0], T) + tuple(src.shape[2:]), dtype=src.dtype, device=src.device)
                pad[:, : blk.T].copy_(src)
                src = pad
            out[name] = masked_rows(src[:, :T], token_mask, None if dense else torch.from_numpy(present), dense)
        return out

    def dense_rows(self, branch_id: Any, layer_idx: int, name: str, T: int, step_idx: int = 0) -> torch.Tensor | None:
        blk = self._caches.get(layer_idx, {}).get((branch_id, step_idx))
        if blk is None or name not in blk.tensors or T > blk.T or not blk.token_present(T).all():
            return None
        return blk.tensors[name][:, :T]

    def has_entry(self, branch_id: Any, layer_idx: int, step_idx: int = 0) -> bool:
        blk = self._caches.get(layer_idx, {}).get((branch_id, step_idx))
        return blk is not None and bool((blk.stamps >= 0).any())

    def touch(self, branch_id: Any, layer_idx: int, selected, T: int, step_idx: int = 0) -> None:
        self._lookup(branch_id, layer_idx, step_idx, T)

    def clear_branch(self, branch_id: Any) -> None:
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
        """Number of cached chunks, optionally for one layer."""
        layers = [self._caches.get(layer_idx, {})] if layer_idx is not None else list(self._caches.values())
        return int(sum(int((b.stamps >= 0).sum()) for layer in layers for b in layer.values()))

    def num_tokens(self, layer_idx: int | None = None) -> int:
        """Number of cached token slots (valid tokens of live chunks)."""
        layers = [self._caches.get(layer_idx, {})] if layer_idx is not None else list(self._caches.values())
        total = 0
        for layer in layers:
            for b in layer.values():
                total += int(b.token_present(b.T).sum())
        return total
