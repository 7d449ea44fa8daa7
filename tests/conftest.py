"""Shared pytest configuration.

Markers:
  gpu -- needs a B200 (sm_100a) and the built libactfold_b200.so; the CPU
         suite runs with ``-m "not gpu"``.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: requires a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    """Load a golden .npz by stem name."""

    def load(name: str):
        return np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False)

    return load


@pytest.fixture(autouse=True)
def _seed():
    np.random.seed(42)
    try:
        import torch

        torch.manual_seed(42)
    except Exception:  # pragma: no cover
        pass
