"""Shared pytest setup: import paths, the `gpu` marker and common fixtures."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "ray-tracing-attention_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device; parity tests of the CUDA path")
    config.addinivalue_line("markers", "slow: longer CPU test")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(GOLDEN / name, allow_pickle=False)
    return load


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))


def ref_bound(actual, expected, tol=3e-6) -> tuple[bool, float, float]:
    """The reference's error_metrics bound: max|a-e| <= tol * max(1, peak|e|)
    (ray_tracing/verification/verify_attention_receipts.py:29-48)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    err = float(np.max(np.abs(a - e), initial=0.0))
    limit = tol * max(1.0, float(np.max(np.abs(e), initial=0.0)))
    return err <= limit, err, limit
