"""Shared fixtures: the `gpu` marker, golden-vector loading and seeded RNGs."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden(name: str) -> dict[str, dict[str, np.ndarray]]:
    """Load tests/golden/<name>.npz grouped by case: {case: {field: array}}."""
    flat = np.load(GOLDEN / f"{name}.npz")
    cases: dict[str, dict[str, np.ndarray]] = {}
    for key in flat.files:
        case, field = key.split("__", 1)
        cases.setdefault(case, {})[field] = flat[key]
    return cases


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    return torch.device("cuda:0")
