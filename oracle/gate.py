"""SimilarityGate restated in numpy (TEST INFRASTRUCTURE: the checker, never the product).

Follows actfold/core/similarity_gate.py:
  * forward            :43-74  (3-D shape checks, parent cast to child dtype, ``sim > tau``)
  * _compute_similarity :76-103 (cosine via F.cosine_similarity, l2, pearson)

Rounding model (reduced-precision inputs). torch evaluates every elementwise op
of a bf16/fp16 tensor in float32 and rounds the result back to the tensor
dtype; reductions accumulate in float32 and round once at the end. For the
cosine metric, ATen's ``cosine_similarity`` (aten/src/ATen/native/Distance.cpp)
computes ``(x1 / clamp_min(||x1||, eps)) * (x2 / clamp_min(||x2||, eps))`` and
sums it, so the chain is:

    n   = rnd(sqrt(sum_f32(x^2)))      per tensor, then max(n, rnd(eps))
    y   = rnd(x / n)                   per element, per tensor
    p   = rnd(y_child * y_parent)      per element (the f32 product is exact)
    sim = rnd(sum_f32(p))

and the Python scalar ``tau`` is converted to the tensor dtype before the
comparison, so ``stable = sim > rnd(tau)``. With float32 inputs every ``rnd``
is the identity.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.numerics import round_to

METRICS = ("cosine", "l2", "pearson")


@dataclass
class GateResult:
    mask: np.ndarray  # bool [B, T], True = stable
    sim: np.ndarray  # float32 [B, T], similarity in the input dtype (bf16 values as f32)
    presum: np.ndarray  # float32 [B, T], the f32 accumulation before the final rounding
    boundary: float  # value of ``presum`` at which the decision flips


def _sum32(x: np.ndarray) -> np.ndarray:
    return np.sum(x, axis=-1, dtype=np.float32)


def _norm(x: np.ndarray, dtype: str) -> np.ndarray:
    return round_to(np.sqrt(_sum32(x * x)), dtype)


def decision_boundary(tau: float, dtype: str) -> float:
    """The f32 pre-rounding similarity at which ``rnd(s) > rnd(tau)`` flips.

    For float32 this is ``tau`` itself. For bf16/fp16 it is the midpoint
    between ``rnd(tau)`` and the next representable value above it.
    """
    t = float(round_to(np.float32(tau), dtype))
    if dtype == "f32":
        return float(np.float32(tau))
    if dtype == "bf16":
        bits = (np.array([t], np.float32).view(np.uint32) >> 16).astype(np.uint32)
        nxt = ((bits + 1) << 16).view(np.float32)[0]
    else:
        nxt = float(np.nextafter(np.float16(t), np.float16(np.inf)))
    return 0.5 * (t + float(nxt))


def gate(
    child: np.ndarray,
    parent: np.ndarray,
    tau: float,
    metric: str = "cosine",
    eps: float = 1e-8,
    dtype: str = "bf16",
) -> GateResult:
    """Per-token similarity and stability mask for [B, T, H] inputs.

    ``child``/``parent`` hold values already representable in ``dtype``.
    """
    if child.ndim != 3 or parent.ndim != 3:
        raise ValueError("SimilarityGate expects 3-D inputs [B, T, H]")
    if child.shape != parent.shape:
        raise ValueError(f"Shape mismatch: h_child {child.shape} vs h_parent {parent.shape}")
    if metric not in METRICS:
        raise ValueError(f"Unsupported metric: {metric}")
    xc = np.asarray(child, np.float32)
    xp = np.asarray(parent, np.float32)
    r = lambda v: round_to(v, dtype)  # noqa: E731
    eps_d = r(np.float32(eps))
    if metric == "cosine":
        nc = np.maximum(_norm(xc, dtype), eps_d)[..., None]
        npar = np.maximum(_norm(xp, dtype), eps_d)[..., None]
        p = r(r(xc / nc) * r(xp / npar))
        presum = _sum32(p)
    elif metric == "l2":
        d = r(xc - xp)
        l2 = _norm(d, dtype)
        denom = np.float32(xc.shape[-1] ** 0.5 + eps)
        presum = np.float32(1.0) - r(l2 / denom)
    else:  # pearson
        H = xc.shape[-1]
        mc = r(_sum32(xc) / np.float32(H))[..., None]
        mp = r(_sum32(xp) / np.float32(H))[..., None]
        cc = r(xc - mc)
        pc = r(xp - mp)
        num = r(_sum32(r(cc * pc)))
        den = r(r(_norm(cc, dtype) * _norm(pc, dtype)) + np.float32(eps))
        presum = num / den
    sim = r(presum)
    t = r(np.float32(tau))
    return GateResult(
        mask=sim > t,
        sim=sim.astype(np.float32),
        presum=np.asarray(presum, np.float32),
        boundary=decision_boundary(tau, dtype),
    )


def exempt_rows(res: GateResult, window: float = 1e-4) -> np.ndarray:
    """Rows whose f32 similarity lies within ``window`` of the decision boundary.

    Only these rows may legitimately disagree between two correct
    implementations that accumulate in a different order.
    """
    return np.abs(res.presum - np.float32(res.boundary)) < window


def compact(mask: np.ndarray) -> tuple[list[np.ndarray], list[np.ndarray], np.ndarray]:
    """Order-preserving stable / divergent index lists per batch row, and divergent counts."""
    stable = [np.nonzero(m)[0].astype(np.int32) for m in mask]
    div = [np.nonzero(~m)[0].astype(np.int32) for m in mask]
    counts = np.array([len(d) for d in div], dtype=np.int32)
    return stable, div, counts
