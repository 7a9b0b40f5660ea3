"""Shared pytest configuration: the `gpu` marker and common fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    gpu_items = [it for it in items if "gpu" in it.keywords]
    if not gpu_items:
        return
    import torch
    if not torch.cuda.is_available():
        skip = pytest.mark.skip(reason="no CUDA device")
        for it in gpu_items:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def kat():
    return dict(np.load(ROOT / "tests" / "golden" / "kat.npz"))


@pytest.fixture(scope="session")
def tiny_golden():
    return dict(np.load(ROOT / "tests" / "golden" / "tiny_model.npz"))


@pytest.fixture(scope="session")
def tiny_blobs():
    from voxcpm2_b200 import synthetic
    from voxcpm2_b200.config import TINY
    return synthetic.model_blobs(TINY, 0)


def close_stats(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    err = float(np.abs(got - want).max()) if got.size else 0.0
    den = float(np.linalg.norm(got) * np.linalg.norm(want))
    cos = float(got @ want / den) if den > 0 else 1.0
    return err, cos


def assert_parity(got, want, atol=2e-2, cos_min=0.999, what=""):
    """The acceptance bar for floating-point results: max-abs <= atol and cosine >= cos_min."""
    err, cos = close_stats(got, want)
    assert err <= atol and cos >= cos_min, f"{what}: max-abs {err:.3e} (<= {atol}), cosine {cos:.6f} (>= {cos_min})"
    return err, cos
