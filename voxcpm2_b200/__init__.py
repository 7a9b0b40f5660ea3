"""B200-native (sm_100a) VoxCPM2 autoregressive patch loop.

The compute lives in ``libvoxcpm2_cuda.so`` (C ABI declared in
include/voxcpm2_cuda.h); this package holds the model description, the
synthetic-workload generator and a thin ctypes mirror of the reference's host
runtime (``run_decoder_with_kv``, ``cfm_sample``, the patch loop).
"""
from .config import BENCH, SMALL, TINY, ModelConfig  # noqa: F401
