"""make_activation_cache (actfold/core/cache_factory.py:20-49)."""

from __future__ import annotations

from typing import Union

from actfold_b200.core.activation_cache import ActivationCache
from actfold_b200.core.chunked_cache import ChunkedActivationCache

ActivationCacheType = Union[ActivationCache, ChunkedActivationCache]


def make_activation_cache(
    max_entries_per_layer: int = 1024,
    device: str = "cuda",
    use_chunked: bool = False,
    chunk_size: int = 64,
) -> ActivationCacheType:
    if use_chunked:
        return ChunkedActivationCache(max_entries_per_layer=max_entries_per_layer, chunk_size=chunk_size, device=device)
    return ActivationCache(max_entries_per_layer=max_entries_per_layer, device=device)
