"""Rounding helpers for the oracle (test infrastructure only).

bf16 values are carried as float32 arrays whose low 16 bits are zero, so all
arithmetic stays in numpy float32 and every rounding point is explicit.
"""

from __future__ import annotations

import numpy as np


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32.

    This is the conversion torch applies when a float32 intermediate is stored
    into a bfloat16 tensor (c10/util/BFloat16.h round_to_nearest_even).
    """
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    bias = ((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    r = ((u + bias) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32(np.nan)
    return out.reshape(np.shape(x))


def round_f16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest fp16 (ties to even); returns float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round to ``dtype`` in {"bf16", "f16", "f32"}; result is float32."""
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype}")


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Return the uint16 bit patterns of bf16-representable float32 values."""
    a = np.ascontiguousarray(round_bf16(x), dtype=np.float32)
    return (a.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    """Inverse of :func:`bf16_bits`."""
    b = np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)
    return b.view(np.float32)
