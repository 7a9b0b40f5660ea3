"""Seeded synthetic weights and inputs for the benchmark workloads.

No VoxCPM2 checkpoint can be loaded here, so every workload runs on random
weights: matrices and biases N(0, 0.02) in fp16 (the reference's exported .bin
files are fp16, export_components.py:404-458), norm gains 1. The normal draws
use inverse-CDF sampling over 65536 equiprobable quantiles, so a 700M-parameter
model is generated in seconds.
Token ids are uniform over the vocabulary; noise and latents are N(0, 1).
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from typing import Dict

import numpy as np

from .config import COMPONENTS, ModelConfig, component_tensors

_CHUNK = 1 << 24
_QUANTILES = {}


def _normal_table(std: float) -> np.ndarray:
    """65536 equiprobable quantiles of N(0, std), rounded to fp16."""
    if std not in _QUANTILES:
        from scipy.special import ndtri
        u = (np.arange(65536, dtype=np.float64) + 0.5) / 65536.0
        _QUANTILES[std] = (ndtri(u) * std).astype(np.float16)
    return _QUANTILES[std]


def _fill_normal(out: np.ndarray, seed: int, std: float) -> None:
    """Fill a flat fp16 array with N(0, std) draws by inverse-CDF sampling: each
    value is the quantile selected by a uniform 16-bit index from a PCG64 stream."""
    table = _normal_table(std).view(np.uint16)
    bits = out.view(np.uint16)
    g = np.random.Generator(np.random.PCG64(seed))
    for a in range(0, out.size, _CHUNK):
        b = min(out.size, a + _CHUNK)
        idx = g.integers(0, 65536, b - a, dtype=np.uint16)
        bits[a:b] = np.take(table, idx, mode="wrap")


def component_blob(cfg: ModelConfig, component: int, seed: int = 0, std: float = 0.02) -> np.ndarray:
    """Flat fp16 blob of one component in the tensor order of config.component_tensors."""
    tensors = component_tensors(cfg, component)
    total = sum(int(np.prod(s)) for _, s, _ in tensors)
    blob = np.empty(total, dtype=np.float16)
    jobs = []
    off = 0
    for idx, (_, shape, kind) in enumerate(tensors):
        n = int(np.prod(shape))
        view = blob[off:off + n]
        if kind == "g":
            view[:] = np.float16(1.0)
        else:
            jobs.append((view, seed * 1_000_003 + component * 10_007 + idx))
        off += n
    _normal_table(std)
    with ThreadPoolExecutor(max_workers=8) as ex:
        list(ex.map(lambda j: _fill_normal(j[0], j[1], std), jobs))
    return blob


def model_blobs(cfg: ModelConfig, seed: int = 0) -> Dict[int, np.ndarray]:
    return {c: component_blob(cfg, c, seed) for c in COMPONENTS}


def token_ids(cfg: ModelConfig, n: int, seed: int = 1) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, cfg.vocab, size=n, dtype=np.int32)


def normal(shape, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
