"""Shared test setup.

Markers: `gpu` tests need a B200 (sm_100) and run with `pytest -m gpu`; everything else
runs on a CPU-only machine. The oracle (oracle/) is test infrastructure: it is imported
here only as the checker.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "llm-engine_b200"))

GOLDEN = os.path.join(REPO, "tests", "golden", "reference_vectors.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu)")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def lib():
    import llme_b200
    llme_b200.load()
    return llme_b200


def close_to(got: np.ndarray, want: np.ndarray, k: int, factor: float = 1.0) -> bool:
    """The reference's GPU/CPU test tolerance (tests/test_cuda.cpp:38-47): every element
    within 1e-5 * max(k, 1) (times `factor`, 2 for the fused cases)."""
    if got.shape != want.shape:
        return False
    tol = 1e-5 * max(k, 1) * factor
    return bool(np.all(np.abs(got.astype(np.float64) - want.astype(np.float64)) <= tol))


def row_rel_err(got: np.ndarray, want: np.ndarray) -> float:
    """max over rows of ||C - C_ref||_inf / ||C_ref row||_2, the path's error metric."""
    g = got.astype(np.float64)
    w = want.astype(np.float64)
    num = np.abs(g - w).max(axis=1)
    den = np.linalg.norm(w, axis=1)
    den = np.where(den == 0, 1.0, den)
    return float((num / den).max()) if g.size else 0.0


def int8_digits(y: np.ndarray):
    """The kernels' int8 digits of y = x * (127 / max|x|) in base 256, computed in fp32 as the
    device does: y ~ t0 + t1 / 256 + t2 / 65536, a second digit of +128 carried into t0."""
    y = np.asarray(y, dtype=np.float32)
    t0 = np.clip(np.rint(y), -127, 127).astype(np.float32)
    r1 = ((y - t0) * np.float32(256)).astype(np.float32)
    g1 = np.rint(r1).astype(np.float32)
    t2 = np.clip(np.rint(((r1 - g1) * np.float32(256)).astype(np.float32)), -128, 127)
    carry = (g1 > 127).astype(np.float32)
    return t0 + carry, g1 - np.float32(256) * carry, t2.astype(np.float32)
