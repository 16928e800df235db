"""Shared fixtures.  `-m gpu` tests need a CUDA device and the built backend;
everything else runs on the CPU (the driver runs `-m "not gpu"` without a GPU)."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA device) and the built backend")
    config.addinivalue_line("markers", "slow: long-running (large synthetic models)")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden():
    return load_golden


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """max |a - b| / max |b| (norm-relative)."""
    return float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30))
