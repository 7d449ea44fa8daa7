"""Stable/divergent merge and cache gather on the CUDA row kernels.

Drop-in for actfold/core/fused_ops.py:206-324. The optional Triton kernel and
the torch fallbacks of the reference are gone: both functions launch
``af_merge_rows`` / ``af_gather_rows_masked`` and require CUDA tensors.
"""

from __future__ import annotations

import torch

from actfold_b200 import _lib


def merge_stable_divergent(parent_ffn: torch.Tensor, child_out: torch.Tensor, stable_mask: torch.Tensor) -> torch.Tensor:
    """``out[b, t] = parent_ffn[b, t] if stable_mask[b, t] else child_out[b, t]``.

    Raises ValueError on incompatible shapes (fused_ops.py:231-244).
    """
    if parent_ffn.ndim != 3 or child_out.ndim != 3:
        raise ValueError(
            f"parent_ffn and child_out must be 3-D [B, T, H], got {parent_ffn.shape} and {child_out.shape}"
        )
    if parent_ffn.shape != child_out.shape:
        raise ValueError(f"Shape mismatch: parent_ffn {parent_ffn.shape} vs child_out {child_out.shape}")
    if stable_mask.ndim != 2 or stable_mask.shape != parent_ffn.shape[:2]:
        raise ValueError(
            f"stable_mask must be 2-D [B, T] matching parent_ffn {parent_ffn.shape[:2]}, got {stable_mask.shape}"
        )
    _lib.require_cuda(parent_ffn, child_out, what="merge_stable_divergent")
    dev = parent_ffn.device
    if child_out.dtype != parent_ffn.dtype:
        # torch.where promotes mixed inputs to the common dtype.
        common = torch.promote_types(parent_ffn.dtype, child_out.dtype)
        parent_ffn, child_out = parent_ffn.to(common), child_out.to(common)
    child_out = child_out.to(dev)
    stable_mask = stable_mask.to(dev, dtype=torch.bool)
    if stable_mask.stride(1) != 1:
        stable_mask = stable_mask.contiguous()
    if parent_ffn.stride(2) != 1:
        parent_ffn = parent_ffn.contiguous()
    if child_out.stride(2) != 1:
        child_out = child_out.contiguous()
    B, T, H = parent_ffn.shape
    out = torch.empty((B, T, H), dtype=parent_ffn.dtype, device=dev)
    es = out.element_size()
    with torch.cuda.device(dev):
        st = _lib.load().af_merge_rows(
            parent_ffn.data_ptr(), parent_ffn.stride(0) * es, parent_ffn.stride(1) * es,
            child_out.data_ptr(), child_out.stride(0) * es, child_out.stride(1) * es,
            stable_mask.data_ptr(), stable_mask.stride(0),
            out.data_ptr(), out.stride(0) * es, out.stride(1) * es,
            B, T, H * es, _lib.stream_ptr(dev),
        )
    _lib.check(st, "merge_stable_divergent")
    return out


def masked_rows(src: torch.Tensor, token_mask: torch.Tensor, present: torch.Tensor | None = None, dense: bool = True) -> torch.Tensor:
    """Zero-filled copy of ``src`` [Bs, T, ...] selected by ``token_mask`` [B, T].

    ``dense`` True: per-(b, t) selection (all tokens cached). ``dense`` False:
    token t is copied to every batch row when present[t] and any row selects it.
    A stored batch of 1 broadcasts over B.
    """
    _lib.require_cuda(src, what="gather_cached_activations")
    B, T = token_mask.shape
    dev = src.device
    if src.shape[1] < T:
        raise ValueError(f"cached sequence {src.shape[1]} shorter than requested {T}")
    Bs = src.shape[0]
    if Bs != B and Bs != 1:
        if Bs > B:
            src = src[:B]
            Bs = B
        else:
            raise RuntimeError(f"cached batch {Bs} cannot be broadcast to requested batch {B}")
    trailing = tuple(src.shape[2:])
    src = src.contiguous()
    row = int(torch.Size(trailing).numel()) if trailing else 1
    es = src.element_size()
    out = torch.empty((B, T) + trailing, dtype=src.dtype, device=dev)
    mask = token_mask.to(dev, dtype=torch.bool).contiguous()
    pres = None if present is None else present.to(dev, dtype=torch.bool).contiguous()
    sb = 0 if Bs == 1 and B > 1 else src.stride(0) * es
    with torch.cuda.device(dev):
        st = _lib.load().af_gather_rows_masked(
            src.data_ptr(), sb, src.stride(1) * es,
            mask.data_ptr(), mask.stride(0), _lib.ptr(pres), 0 if dense else 1,
            out.data_ptr(), out.stride(0) * es, out.stride(1) * es,
            B, T, row * es, _lib.stream_ptr(dev),
        )
    _lib.check(st, "gather_cached_activations")
    return out


def gather_cached_activations(cache, branch_id, layer_idx: int, token_mask: torch.Tensor, step_idx: int = 0) -> dict[str, torch.Tensor]:
    """Reconstruct ``[B, T, ...]`` activations; unselected or missing tokens are zero.

    ``cache`` is either an :class:`~actfold_b200.core.activation_cache.ActivationCache`
    layer store or the reference's raw per-token mapping
    ``{(branch, layer, token, step): {name: Tensor[B, ...]}}``. Raises KeyError when
    token 0 is missing (fused_ops.py:288-289).
    """
    from actfold_b200.core.activation_cache import ActivationCache

    if isinstance(cache, ActivationCache):
        return cache.get(branch_id, layer_idx, token_mask, step_idx)
    B, T = token_mask.shape
    k0 = (branch_id, layer_idx, 0, step_idx)
    if k0 not in cache:
        raise KeyError(f"No cache entry for branch={branch_id}, layer={layer_idx}, step={step_idx}")
    sample = cache[k0]
    present_list = [(branch_id, layer_idx, t, step_idx) in cache for t in range(T)]
    dense = all(present_list)
    out: dict[str, torch.Tensor] = {}
    for name, s in sample.items():
        rows = []
        for t in range(T):
            key = (branch_id, layer_idx, t, step_idx)
            rows.append(cache[key][name] if key in cache else torch.zeros_like(s))
        stacked = torch.stack(rows, dim=1)  # assemble the per-token entries into one block
        present = None if dense else torch.tensor(present_list, dtype=torch.bool, device=stacked.device)
        out[name] = masked_rows(stacked, token_mask, present, dense)
    return out
