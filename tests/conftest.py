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
    config.addinivalue_line("markers", "slow: full-size CPU oracle runs")


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
