"""ctypes mirror of the reference host runtime over libvoxcpm2_cuda.so.

Names follow the reference: ``Stream.decoder_step`` is run_decoder_with_kv
(src/kvcache.cpp:232-279), ``Stream.cfm_sample`` is cfm_sample
(src/synthesizer.cpp:86-170), ``Stream.generate`` is generate_with_caches
without the audio VAE, ``sdpa`` is the VoxCPM2SDPA layer's forward. Errors
raise ``VxcError`` carrying the vxc_status code, as the reference's C ABI maps
exceptions to voxcpm2_status (src/c_api.cpp:168-193).

There is no CPU path: loading fails loudly when the CUDA library has not been
built, and every call needs a CUDA device.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import Callable, Dict, Optional

import numpy as np

from .config import ModelConfig, component_count

LIB_PATH = Path(__file__).resolve().parent / "libvoxcpm2_cuda.so"

STATUS = {0: "OK", 1: "INVALID_ARGUMENT", 2: "INVALID_STATE", 3: "CANCELLED", 4: "OUT_OF_MEMORY",
          5: "RUNTIME_ERROR"}
BASE, RESIDUAL = 0, 1
PLAN_THROUGHPUT, PLAN_LATENCY = 0, 1  # vxc_stream_set_plan


class VxcError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class Desc(C.Structure):
    _fields_ = [
        ("hidden", C.c_int32), ("ffn", C.c_int32), ("q_heads", C.c_int32), ("kv_heads", C.c_int32),
        ("head_dim", C.c_int32), ("base_layers", C.c_int32), ("res_layers", C.c_int32),
        ("dit_hidden", C.c_int32), ("dit_ffn", C.c_int32), ("dit_layers", C.c_int32),
        ("dit_q_heads", C.c_int32), ("dit_kv_heads", C.c_int32), ("feat_dim", C.c_int32),
        ("patch_size", C.c_int32), ("vocab", C.c_int32), ("fsq_dim", C.c_int32),
        ("fsq_scale", C.c_float), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("rope_original_max", C.c_int32), ("base_residual_scale", C.c_float),
        ("res_residual_scale", C.c_float), ("dit_residual_scale", C.c_float),
        ("embed_scale", C.c_float), ("audio_start_token", C.c_int32),
        ("max_generation_patches", C.c_int32),
    ]


class StreamState(C.Structure):
    _fields_ = [("kv_len", C.c_int32 * 2), ("patches", C.c_int32), ("stopped", C.c_int32),
                ("stop_logits", C.c_float * 2), ("prefix_len", C.c_int32), ("error", C.c_int32),
                ("graph_kernels", C.c_int32)]


PROFILE_KERNELS = {"dit_gateup": 0, "dit_down": 1, "dit_qkv": 2, "base_gateup": 3, "base_down": 4,
                   "base_qkv": 5, "base_attn": 6, "dit_o": 7, "base_step": 9, "res_step": 10,
                   "dit_eval": 11}


PROGRESS_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_int32, C.c_int32)

# exported name -> (argtypes, restype)
SIGNATURES = None
_lib = None


def _signatures():
    vp, i, f, u = C.c_void_p, C.c_int32, C.c_float, C.c_uint32
    return {
        "vxc_abi_version": ([], u),
        "vxc_last_error": ([], C.c_char_p),
        "vxc_component_weight_count": ([C.POINTER(Desc), i], C.c_size_t),
        "vxc_device_create": ([i, C.POINTER(Desc), C.POINTER(vp)], i),
        "vxc_device_destroy": ([vp], None),
        "vxc_load_weights": ([vp, i, vp, C.c_size_t], i),
        "vxc_set_rope_factors": ([vp, vp, vp, i], i),
        "vxc_stream_create": ([vp, i, C.POINTER(vp)], i),
        "vxc_stream_destroy": ([vp], None),
        "vxc_stream_reset": ([vp], i),
        "vxc_stream_set_plan": ([vp, i], i),
        "vxc_stream_cancel": ([vp], None),
        "vxc_token_count": ([vp, i, C.POINTER(i)], i),
        "vxc_read_cache": ([vp, i, i, vp, vp], i),
        "vxc_decoder_step": ([vp, i, vp, i, vp], i),
        "vxc_text_embed": ([vp, vp, i, vp], i),
        "vxc_run_component": ([vp, i, vp, vp, vp], i),
        "vxc_dit_estimator": ([vp, vp, vp, vp, vp, vp, vp], i),
        "vxc_cfm_sample": ([vp, vp, vp, vp, i, f, vp], i),
        "vxc_prefill": ([vp, vp, i], i),
        "vxc_prefill_rows": ([vp, vp, vp, vp, i], i),
        "vxc_patch_step": ([vp, vp, i, i, f, i, vp, C.POINTER(i)], i),
        "vxc_generate": ([vp, vp, i, i, i, f, i, u, vp, C.POINTER(i), vp, vp, vp, PROGRESS_FN, vp], i),
        "vxc_sdpa": ([vp, i, i, i, vp, vp, i, i, i, vp, i, vp, vp, i, f, vp, vp, vp, vp], i),
        "vxc_sdpa_host": ([vp, i, i, i, vp, vp, i, i, i, vp, i, vp, vp, i, f, vp, vp, vp], i),
        "vxc_sdpa_decode_noalloc": ([vp, i, i, vp, vp, i, i, vp, vp, vp, i, f, vp, vp, vp, vp], i),
        "vxc_timestep_embedding": ([vp, i, i, f, f, i, vp], i),
        "vxc_upload_noise": ([vp, vp, i], i),
        "vxc_patch_step_async": ([vp, i, f, i], i),
        "vxc_stream_synchronize": ([vp], i),
        "vxc_patch_submit": ([vp, vp, i, f, i], i),
        "vxc_patch_collect": ([vp, vp, C.POINTER(i)], i),
        "vxc_patch_run": ([C.POINTER(vp), i, vp, i, i, f, i, vp, vp], i),
        "vxc_read_state": ([vp, C.POINTER(StreamState)], i),
        "vxc_read_hidden": ([vp, vp, vp], i),
        "vxc_read_latents": ([vp, i, i, vp], i),
        "vxc_profile_kernel": ([vp, i, i, C.POINTER(f), C.POINTER(C.c_double)], i),
        "vxc_profile_kernel_concurrent": ([C.POINTER(vp), i, i, i, C.POINTER(f), C.POINTER(C.c_double)], i),
        "vxc_stream_cuda_handle": ([vp, C.POINTER(vp)], i),
        "vxc_group_create": ([vp, i, i, C.POINTER(vp)], i),
        "vxc_group_destroy": ([vp], None),
        "vxc_group_stream": ([vp, i, C.POINTER(vp)], i),
        "vxc_group_patch_step_async": ([vp, i, f, i], i),
        "vxc_group_synchronize": ([vp], i),
        "vxc_group_graph_kernels": ([vp, C.POINTER(i)], i),
    }


def lib() -> C.CDLL:
    global _lib, SIGNATURES
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built: run `python -m voxcpm2_b200.build` (no CPU fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        SIGNATURES = _signatures()
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise VxcError(rc, lib().vxc_last_error().decode(errors="replace"))


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def desc(cfg: ModelConfig) -> Desc:
    d = Desc()
    for name, _ in Desc._fields_:
        setattr(d, name, getattr(cfg, name))
    return d


class Device:
    """A model loaded on one CUDA device (weights shared by its streams)."""

    def __init__(self, cfg: ModelConfig, device: int = 0, blobs: Optional[Dict[int, np.ndarray]] = None):
        self.cfg = cfg
        self._desc = desc(cfg)
        h = C.c_void_p()
        _check(lib().vxc_device_create(device, C.byref(self._desc), C.byref(h)))
        self._h = h
        if blobs:
            for comp, blob in blobs.items():
                self.load(comp, blob)

    def load(self, component: int, blob: np.ndarray) -> None:
        blob = np.ascontiguousarray(blob, dtype=np.float16)
        if blob.size != component_count(self.cfg, component):
            raise ValueError(f"component {component}: {blob.size} values, expected {component_count(self.cfg, component)}")
        _check(lib().vxc_load_weights(self._h, component, _p(blob), blob.size))

    def set_rope_factors(self, short_factor, long_factor=None) -> None:
        """The base decoder's LongRoPE factors (model.json setting.rope.short_factor /
        long_factor, at least head_dim / 2 values each; long optional). Streams pick them up at
        their next prefill, decoder step or patch step."""
        sf = np.ascontiguousarray(short_factor, dtype=np.float32)
        lf = None if long_factor is None else np.ascontiguousarray(long_factor, dtype=np.float32)
        _check(lib().vxc_set_rope_factors(self._h, _p(sf), _p(lf) if lf is not None else None, sf.size))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().vxc_device_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: module globals may already be gone
            pass


class Stream:
    """One synthesis stream: KV caches for both decoders plus its CUDA graph."""

    def __init__(self, device: Device, kv_capacity: int = 1024):
        self.dev = device
        self.cfg = device.cfg
        self.cap = kv_capacity
        h = C.c_void_p()
        _check(lib().vxc_stream_create(device._h, kv_capacity, C.byref(h)))
        self._h = h
        self._owned = True

    @classmethod
    def _member(cls, device: Device, handle: C.c_void_p, kv_capacity: int) -> "Stream":
        """A view of a stream owned by a Group (closing it does not free it)."""
        st = cls.__new__(cls)
        st.dev = device
        st.cfg = device.cfg
        st.cap = kv_capacity
        st._h = handle
        st._owned = False
        return st

    def close(self) -> None:
        if getattr(self, "_h", None):
            if self._owned:
                lib().vxc_stream_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: module globals may already be gone
            pass

    def set_plan(self, plan: int) -> None:
        """PLAN_THROUGHPUT (the default) or PLAN_LATENCY for a stream that runs alone;
        takes effect at the next patch."""
        _check(lib().vxc_stream_set_plan(self._h, plan))

    # -- KV cache runner ---------------------------------------------------
    def reset(self) -> None:
        _check(lib().vxc_stream_reset(self._h))

    def cancel(self) -> None:
        lib().vxc_stream_cancel(self._h)

    def token_count(self, which: int) -> int:
        n = C.c_int32()
        _check(lib().vxc_token_count(self._h, which, C.byref(n)))
        return n.value

    def read_cache(self, which: int, layer: int):
        t = self.token_count(which)
        k = np.empty((self.cfg.kv_heads, t, self.cfg.head_dim), np.float32)
        v = np.empty_like(k)
        _check(lib().vxc_read_cache(self._h, which, layer, _p(k), _p(v)))
        return k, v

    def decoder_step(self, which: int, embed) -> np.ndarray:
        embed = _f32(embed).reshape(-1, self.cfg.hidden)
        out = np.empty_like(embed)
        _check(lib().vxc_decoder_step(self._h, which, _p(embed), embed.shape[0], _p(out)))
        return out

    # -- small graphs ------------------------------------------------------
    def text_embed(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.cfg.hidden), np.float32)
        _check(lib().vxc_text_embed(self._h, _p(ids), ids.size, _p(out)))
        return out

    def run_component(self, component: int, in0, in1=None) -> np.ndarray:
        n = {3: self.cfg.hidden, 4: self.cfg.hidden, 5: 2 * self.cfg.dit_hidden, 6: 2, 7: self.cfg.hidden}[component]
        out = np.empty(n, np.float32)
        a = _f32(in0)
        b = None if in1 is None else _f32(in1)
        _check(lib().vxc_run_component(self._h, component, _p(a), _p(b), _p(out)))
        return out

    # -- CFM ----------------------------------------------------------------
    def dit_estimator(self, x_in, mu_in, t_in, cond_in, dt_in) -> np.ndarray:
        out = np.empty((2, self.cfg.latent), np.float32)
        _check(lib().vxc_dit_estimator(self._h, _p(_f32(x_in)), _p(_f32(mu_in)), _p(_f32(t_in)),
                                       _p(_f32(cond_in)), _p(_f32(dt_in)), _p(out)))
        return out

    def cfm_sample(self, mu, cond, noise, timesteps: int = 10, cfg_value: float = 2.0) -> np.ndarray:
        out = np.empty(self.cfg.latent, np.float32)
        _check(lib().vxc_cfm_sample(self._h, _p(_f32(mu)), _p(_f32(cond)), _p(_f32(noise)), timesteps,
                                    cfg_value, _p(out)))
        return out

    # -- patch loop --------------------------------------------------------
    def prefill(self, text_ids) -> None:
        ids = np.ascontiguousarray(text_ids, dtype=np.int32)
        _check(lib().vxc_prefill(self._h, _p(ids), ids.size))

    def prefill_rows(self, token_ids, is_audio=None, audio_latents=None) -> None:
        """Prefix given row by row: token ids, is_audio flags (None: all text) and the
        audio rows' latent patches in row order ([n_audio][D*P], d-major)."""
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        flags = None if is_audio is None else np.ascontiguousarray(is_audio, dtype=np.int32)
        if flags is not None and flags.shape != ids.shape:
            raise ValueError("one is_audio flag per row")
        lat = None if audio_latents is None else _f32(audio_latents).reshape(-1, self.cfg.latent)
        _check(lib().vxc_prefill_rows(self._h, _p(ids), _p(flags), _p(lat), ids.size))

    def patch_step(self, noise, min_patches: int, step: int, cfg_value: float = 2.0, timesteps: int = 10,
                   out=None):
        """One synchronous patch step: (latent, stop). out: an optional float32 [D*P]
        array that receives the latent; a C-contiguous float32 noise array is passed
        without a copy."""
        lat = np.empty(self.cfg.latent, np.float32) if out is None else out
        if not (lat.dtype == np.float32 and lat.flags.c_contiguous and lat.size == self.cfg.latent):
            raise ValueError("out must be a contiguous float32 array of one latent patch")
        if noise is not None and not (isinstance(noise, np.ndarray) and noise.dtype == np.float32
                                      and noise.flags.c_contiguous):
            noise = _f32(noise)
        stop = C.c_int32(0)
        rc = lib().vxc_patch_step(self._h, None if noise is None else noise.ctypes.data, min_patches, step,
                                  cfg_value, timesteps, lat.ctypes.data, C.byref(stop))
        if rc:
            _check(rc)
        return lat, bool(stop.value)

    def generate(self, text_ids, min_patches: int = 2, timesteps: int = 10, cfg_value: float = 2.0,
                 max_patches_override: int = 0, seed: int = 0, trace: bool = True,
                 progress: Optional[Callable[[int, int], bool]] = None) -> dict:
        ids = np.ascontiguousarray(text_ids, dtype=np.int32)
        cap = min(self.cfg.max_generation_patches, int(max(1, ids.size) * 6.0 + 10.0))
        if max_patches_override > 0:
            cap = min(cap, max_patches_override)
        lat = np.zeros((cap, self.cfg.latent), np.float32)
        lm = np.zeros((cap, self.cfg.hidden), np.float32) if trace else None
        res = np.zeros((cap, self.cfg.hidden), np.float32) if trace else None
        stop = np.zeros((cap, 2), np.float32) if trace else None
        n = C.c_int32(0)
        cb = PROGRESS_FN(lambda _u, done, total: 1 if progress(done, total) else 0) if progress else PROGRESS_FN()
        _check(lib().vxc_generate(self._h, _p(ids), ids.size, min_patches, timesteps, cfg_value,
                                  max_patches_override, seed, _p(lat), C.byref(n), _p(lm), _p(res), _p(stop),
                                  cb, None))
        k = n.value
        out = {"patches": k, "latents": lat[:k]}
        if trace:
            out.update(lm_hidden=lm[:k], res_hidden=res[:k], stop_logits=stop[:k])
        return out

    # -- device-resident driving -----------------------------------------
    def upload_noise(self, noise) -> None:
        noise = _f32(noise).reshape(-1, self.cfg.latent)
        _check(lib().vxc_upload_noise(self._h, _p(noise), noise.shape[0]))

    def patch_step_async(self, min_patches: int, cfg_value: float = 2.0, timesteps: int = 10) -> None:
        _check(lib().vxc_patch_step_async(self._h, min_patches, cfg_value, timesteps))

    def synchronize(self) -> None:
        _check(lib().vxc_stream_synchronize(self._h))

    def patch_submit(self, noise, min_patches: int, cfg_value: float = 2.0, timesteps: int = 10) -> None:
        """Queue one patch step (host noise) without waiting; see patch_collect. A
        C-contiguous float32 noise array is passed without a copy."""
        if not (isinstance(noise, np.ndarray) and noise.dtype == np.float32 and noise.flags.c_contiguous):
            noise = _f32(noise)
        rc = _lib.vxc_patch_submit(self._h, noise.ctypes.data, min_patches, cfg_value, timesteps)
        if rc:
            _check(rc)

    def patch_collect(self, out=None):
        """(latent, stop) of the oldest queued patch, waiting for that patch only.
        out: an optional float32 [D*P] array that receives the latent."""
        lat = np.empty(self.cfg.latent, np.float32) if out is None else out
        if not (lat.dtype == np.float32 and lat.flags.c_contiguous and lat.size == self.cfg.latent):
            raise ValueError("out must be a contiguous float32 array of one latent patch")
        stop = C.c_int32(0)
        rc = _lib.vxc_patch_collect(self._h, lat.ctypes.data, C.byref(stop))
        if rc:
            _check(rc)
        return lat, bool(stop.value)

    def state(self) -> StreamState:
        st = StreamState()
        _check(lib().vxc_read_state(self._h, C.byref(st)))
        return st

    def hidden(self):
        lm = np.empty(self.cfg.hidden, np.float32)
        res = np.empty(self.cfg.hidden, np.float32)
        _check(lib().vxc_read_hidden(self._h, _p(lm), _p(res)))
        return lm, res

    def latents(self, first: int, count: int) -> np.ndarray:
        out = np.empty((count, self.cfg.latent), np.float32)
        _check(lib().vxc_read_latents(self._h, first, count, _p(out)))
        return out

    def profile_kernel(self, kernel: str, iters: int = 50):
        """(ms per launch, algorithmic bytes per launch) of one hot kernel, timed as
        'iters' graph-captured launches cycling through the layers."""
        ms = C.c_float()
        nb = C.c_double()
        _check(lib().vxc_profile_kernel(self._h, PROFILE_KERNELS[kernel], iters, C.byref(ms), C.byref(nb)))
        return float(ms.value), float(nb.value)

    @staticmethod
    def profile_kernel_concurrent(streams, kernel: str, iters: int = 100):
        """(ms for the whole set, algorithmic bytes per launch): the kernel's graph of
        'iters' launches replayed on every stream at once."""
        arr = (C.c_void_p * len(streams))(*[st._h for st in streams])
        ms = C.c_float()
        nb = C.c_double()
        _check(lib().vxc_profile_kernel_concurrent(arr, len(streams), PROFILE_KERNELS[kernel], iters, C.byref(ms),
                                                   C.byref(nb)))
        return float(ms.value), float(nb.value)

    def cuda_stream(self) -> int:
        h = C.c_void_p()
        _check(lib().vxc_stream_cuda_handle(self._h, C.byref(h)))
        return h.value or 0


def patch_run(streams, noise, min_patches: int, cfg_value: float = 2.0, timesteps: int = 10, out=None):
    """vxc_patch_run: the patch loop of several streams driven from this thread in
    native code. noise [n][patches][D*P] float32; returns (latents [n][patches][D*P],
    patches run per stream). out: an optional float32 array of the latents' shape."""
    n = len(streams)
    if not (isinstance(noise, np.ndarray) and noise.dtype == np.float32 and noise.flags.c_contiguous):
        noise = _f32(noise)
    patches = noise.shape[1]
    lat = np.empty(noise.shape, np.float32) if out is None else out
    if lat.shape != noise.shape or lat.dtype != np.float32 or not lat.flags.c_contiguous:
        raise ValueError("out must be a contiguous float32 array shaped like noise")
    counts = np.zeros(n, np.int32)
    arr = (C.c_void_p * n)(*[st._h for st in streams])
    rc = _lib.vxc_patch_run(arr, n, noise.ctypes.data, patches, min_patches, cfg_value, timesteps, lat.ctypes.data,
                            counts.ctypes.data)
    if rc:
        _check(rc)
    return lat, counts


class Group:
    """Up to 8 streams stepped together: one CUDA graph per group patch, with the
    estimator evaluations of all members batched into one pass over the DiT
    weights. Members are ordinary streams (prefill, noise, state, latents)."""

    def __init__(self, device: Device, n_streams: int, kv_capacity: int = 1024):
        self.dev = device
        h = C.c_void_p()
        _check(lib().vxc_group_create(device._h, n_streams, kv_capacity, C.byref(h)))
        self._h = h
        self.streams = []
        for m in range(n_streams):
            sh = C.c_void_p()
            _check(lib().vxc_group_stream(self._h, m, C.byref(sh)))
            self.streams.append(Stream._member(device, sh, kv_capacity))

    def patch_step_async(self, min_patches: int, cfg_value: float = 2.0, timesteps: int = 10) -> None:
        _check(lib().vxc_group_patch_step_async(self._h, min_patches, cfg_value, timesteps))

    def synchronize(self) -> None:
        _check(lib().vxc_group_synchronize(self._h))

    def graph_kernels(self) -> int:
        n = C.c_int32()
        _check(lib().vxc_group_graph_kernels(self._h, C.byref(n)))
        return int(n.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            for st in self.streams:
                st._h = None
            lib().vxc_group_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: module globals may already be gone
            pass


def sdpa(q, k, v, mask=None, past_k=None, past_v=None, scale: float = 0.0, want_cache: bool = False):
    """VoxCPM2SDPA forward on host arrays (ncnn layout), computed on the GPU."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    heads, src, d = q.shape
    groups, cur, dv = v.shape
    past = 0 if past_k is None else past_k.shape[1]
    m = None if mask is None else _f32(mask)
    mask_c = 0 if m is None else (m.shape[0] if m.ndim == 3 else 1)
    pk = None if past_k is None else _f32(past_k)
    pv = None if past_v is None else _f32(past_v)
    out = np.empty((heads, src, dv), np.float32)
    ok = np.empty((groups, past + cur, d), np.float32) if want_cache else None
    ov = np.empty((groups, past + cur, dv), np.float32) if want_cache else None
    _check(lib().vxc_sdpa_host(_p(q), heads, src, d, _p(k), _p(v), groups, cur, dv, _p(m), mask_c, _p(pk), _p(pv),
                               past, float(scale), _p(out), _p(ok), _p(ov)))
    return (out, ok, ov) if want_cache else out


def sdpa_device(q_ptr: int, heads: int, src: int, d: int, k_ptr: int, v_ptr: int, groups: int, cur: int, dv: int,
                mask_ptr: int, mask_c: int, pk_ptr: int, pv_ptr: int, past: int, scale: float, out_ptr: int,
                ok_ptr: int = 0, ov_ptr: int = 0, stream: int = 0) -> None:
    """vxc_sdpa on device pointers (e.g. torch tensors' data_ptr()); asynchronous on 'stream'."""
    _check(lib().vxc_sdpa(q_ptr, heads, src, d, k_ptr, v_ptr, groups, cur, dv, mask_ptr or None, mask_c,
                          pk_ptr or None, pv_ptr or None, past, scale, out_ptr, ok_ptr or None, ov_ptr or None,
                          stream or None))


def sdpa_decode_noalloc(q_ptr: int, heads: int, d: int, k_ptr: int, v_ptr: int, groups: int, cur: int,
                        mask_ptr: int, pk_ptr: int, pv_ptr: int, past: int, scale: float, out_ptr: int,
                        ok_ptr: int = 0, ov_ptr: int = 0, stream: int = 0) -> None:
    """vxc_sdpa_decode_noalloc on device pointers: one query row, no device allocation
    (its scratch is a fixed array inside the library); asynchronous on 'stream'."""
    _check(lib().vxc_sdpa_decode_noalloc(q_ptr, heads, d, k_ptr, v_ptr, groups, cur, mask_ptr or None,
                                         pk_ptr or None, pv_ptr or None, past, scale, out_ptr, ok_ptr or None,
                                         ov_ptr or None, stream or None))


def timestep_embedding(inp, half_dim: int = 512, scale: float = 1000.0, max_period: float = 10000.0,
                       schedule_mode: int = 0) -> np.ndarray:
    """VoxCPM2TimestepEmbedding forward on host arrays, computed on the GPU: [n][2 * half_dim]."""
    x = _f32(inp).ravel()
    out = np.empty((x.size, 2 * half_dim), np.float32)
    _check(lib().vxc_timestep_embedding(_p(x), x.size, half_dim, float(scale), float(max_period), schedule_mode,
                                        _p(out)))
    return out
