"""Seeded synthetic weights and inputs for the benchmark workloads.

No VoxCPM2 checkpoint can be loaded here, so every workload runs on random
weights: matrices and biases N(0, 0.02) rounded to fp16 (the reference's
exported .bin files are fp16, export_components.py:404-458), norm gains 1.
Token ids are uniform over the vocabulary; noise and latents are N(0, 1).
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from typing import Dict

import numpy as np

from .config import COMPONENTS, ModelConfig, component_tensors

_CHUNK = 1 << 22


def _fill_normal(out: np.ndarray, seed: int, std: float) -> None:
    """Fill a flat fp16 array with N(0, std) draws, chunk-parallel and deterministic."""
    n = out.size
    chunks = [(i, min(n, i + _CHUNK)) for i in range(0, n, _CHUNK)]
    ss = np.random.SeedSequence(seed)
    seeds = ss.spawn(len(chunks))

    def work(k: int) -> None:
        a, b = chunks[k]
        g = np.random.Generator(np.random.PCG64(seeds[k]))
        vals = g.standard_normal(b - a, dtype=np.float32)
        vals *= np.float32(std)
        out[a:b] = vals.astype(np.float16)

    with ThreadPoolExecutor(max_workers=8) as ex:
        list(ex.map(work, range(len(chunks))))


def component_blob(cfg: ModelConfig, component: int, seed: int = 0, std: float = 0.02) -> np.ndarray:
    """Flat fp16 blob of one component in the tensor order of config.component_tensors."""
    tensors = component_tensors(cfg, component)
    total = sum(int(np.prod(s)) for _, s, _ in tensors)
    blob = np.empty(total, dtype=np.float16)
    off = 0
    for idx, (_, shape, kind) in enumerate(tensors):
        n = int(np.prod(shape))
        view = blob[off:off + n]
        if kind == "g":
            view[:] = np.float16(1.0)
        else:
            _fill_normal(view, seed * 1_000_003 + component * 10_007 + idx, std)
        off += n
    return blob


def model_blobs(cfg: ModelConfig, seed: int = 0) -> Dict[int, np.ndarray]:
    return {c: component_blob(cfg, c, seed) for c in COMPONENTS}


def token_ids(cfg: ModelConfig, n: int, seed: int = 1) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, cfg.vocab, size=n, dtype=np.int32)


def normal(shape, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
