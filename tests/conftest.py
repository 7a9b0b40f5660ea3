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


def fsq_codes_from_hidden(cfg, blobs, lm):
    """The FSQ codes behind LM hidden states. An FSQ output is out_proj(codes / scale)
    (+ bias) with integer codes, so least squares over out_proj's fsq_dim columns
    recovers codes / scale; returns the rounded codes [rows][fsq_dim] and the largest
    distance of the solution from those integers (near 0 for a real FSQ output)."""
    from voxcpm2_b200.config import FSQ
    H, Q = cfg.hidden, cfg.fsq_dim
    b = np.asarray(blobs[FSQ], dtype=np.float16).astype(np.float64)
    out_w = b[Q * H + Q: Q * H + Q + H * Q].reshape(H, Q)
    out_b = b[Q * H + Q + H * Q: Q * H + Q + H * Q + H]
    lm = np.atleast_2d(np.asarray(lm, np.float64))
    sol, *_ = np.linalg.lstsq(out_w, (lm - out_b).T, rcond=None)
    x = sol.T * cfg.fsq_scale
    codes = np.rint(x)
    return codes.astype(np.float32), float(np.abs(x - codes).max()) if x.size else 0.0


def fsq_forced_disagreements(fsq_pre, codes):
    """Codes that differ from the oracle's own rounding of its pre-rounding values:
    [(patch, index, own code, forced code, distance of the value from the boundary
    between the two codes)]."""
    own = np.rint(fsq_pre[: codes.shape[0]])
    out = []
    for p, j in zip(*np.nonzero(own != codes)):
        v, c = float(fsq_pre[p, j]), float(codes[p, j])
        boundary = 0.5 * (float(own[p, j]) + c)
        out.append((int(p), int(j), float(own[p, j]), c, abs(v - boundary)))
    return out
