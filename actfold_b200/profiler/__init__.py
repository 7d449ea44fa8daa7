"""Stability profiling (drop-in for ``actfold.profiler.stability_profiler``)."""

from actfold_b200.profiler.stability_profiler import (
    GLOBAL_STABILITY_PROFILER,
    LayerStabilityStats,
    StabilityProfile,
    StabilityProfiler,
)

__all__ = ["GLOBAL_STABILITY_PROFILER", "LayerStabilityStats", "StabilityProfile", "StabilityProfiler"]
