"""ctypes binding of the CPU oracle (oracle.cpp) -- test infrastructure only.

Every function mirrors one reference routine; see oracle.h for the file:line
each follows. Arrays are numpy float32 (C order) unless stated otherwise.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path
from typing import Dict, Optional

import numpy as np

from voxcpm2_b200.config import ModelConfig, component_count

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liborc.so"
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


class _Desc(C.Structure):
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


def build(force: bool = False) -> Path:
    """Compile oracle.cpp with its Makefile (plain g++, OpenMP)."""
    src = _HERE / "oracle.cpp"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(_LIB_PATH))
        _setup(_lib)
        set_threads(int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1)))
    return _lib


def _setup(L) -> None:
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    L.orc_set_threads.argtypes = [i]
    L.orc_get_threads.restype = i
    L.orc_sdpa.argtypes = [vp, i, i, i, vp, vp, i, i, i, vp, i, vp, vp, i, f, vp, vp, vp]
    L.orc_sdpa.restype = i
    L.orc_timestep_embedding.argtypes = [vp, i, i, f, f, i, vp]
    L.orc_decoder_mask.argtypes = [i, i, vp]
    L.orc_rope_cache.argtypes = [i, f, i, vp, vp, i, i, vp, vp]
    L.orc_sway_t_span.argtypes = [i, vp]
    L.orc_zero_init_steps.argtypes = [i]
    L.orc_zero_init_steps.restype = i
    L.orc_optimized_scale.argtypes = [vp, vp, i]
    L.orc_optimized_scale.restype = f
    L.orc_max_patches.argtypes = [i, i]
    L.orc_max_patches.restype = i
    L.orc_noise_table.argtypes = [C.c_uint32, i, i, vp]
    L.orc_model_create.argtypes = [C.POINTER(_Desc)]
    L.orc_model_create.restype = vp
    L.orc_model_destroy.argtypes = [vp]
    L.orc_component_count.argtypes = [C.POINTER(_Desc), i]
    L.orc_component_count.restype = C.c_size_t
    L.orc_set_weights.argtypes = [vp, i, vp, C.c_size_t]
    L.orc_set_weights.restype = i
    L.orc_set_rope_factors.argtypes = [vp, vp, vp, i]
    L.orc_set_rope_factors.restype = i
    L.orc_reset_caches.argtypes = [vp]
    L.orc_token_count.argtypes = [vp, i]
    L.orc_token_count.restype = i
    L.orc_read_cache.argtypes = [vp, i, i, vp, vp]
    L.orc_read_cache.restype = i
    L.orc_decoder_forward.argtypes = [vp, i, vp, i, vp, vp, vp, vp]
    L.orc_decoder_forward.restype = i
    L.orc_text_embed.argtypes = [vp, vp, i, vp]
    L.orc_text_embed.restype = i
    L.orc_fsq.argtypes = [vp, vp, i, vp]
    L.orc_fsq.restype = i
    L.orc_fusion_proj.argtypes = [vp, vp, vp, i, vp]
    L.orc_fusion_proj.restype = i
    L.orc_dit_proj.argtypes = [vp, vp, vp, vp]
    L.orc_dit_proj.restype = i
    L.orc_stop_head.argtypes = [vp, vp, vp]
    L.orc_stop_head.restype = i
    L.orc_feat_encoder.argtypes = [vp, vp, vp]
    L.orc_feat_encoder.restype = i
    L.orc_dit_estimator.argtypes = [vp, vp, vp, vp, vp, vp, vp]
    L.orc_dit_estimator.restype = i
    L.orc_cfm_sample.argtypes = [vp, vp, vp, vp, i, f, vp]
    L.orc_cfm_sample.restype = i
    L.orc_generate.argtypes = [vp, vp, i, i, i, f, i, C.c_uint32, vp, vp, vp, vp, C.POINTER(C.c_int)]
    L.orc_generate.restype = i
    L.orc_generate_rows.argtypes = [vp, vp, vp, vp, i, i, i, i, f, i, C.c_uint32, vp, vp, vp, vp, C.POINTER(C.c_int)]
    L.orc_generate_rows.restype = i
    L.orc_trace_fsq.argtypes = [vp, vp, i]
    L.orc_trace_fsq.restype = i
    L.orc_force_fsq.argtypes = [vp, vp, i]
    L.orc_force_fsq.restype = i


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return lib().orc_get_threads()


def desc(cfg: ModelConfig) -> _Desc:
    d = _Desc()
    for name, _ in _Desc._fields_:
        setattr(d, name, getattr(cfg, name))
    return d


# ----------------------------------------------------------- per-op ------
def sdpa(q, k, v, mask=None, past_k=None, past_v=None, scale: float = 0.0, want_cache: bool = False):
    """VoxCPM2SDPA CPU forward. q [heads][src][d]; k/v [groups][cur][d]; mask [src][dst]
    or [heads][src][dst]; past_k/v [groups][past][d]. Returns out (and new k/v)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    heads, src, d = q.shape
    groups, cur, dv = v.shape
    past = 0 if past_k is None else past_k.shape[1]
    pk = None if past_k is None else _f32(past_k)
    pv = None if past_v is None else _f32(past_v)
    m = None if mask is None else _f32(mask)
    mask_c = 0 if m is None else (m.shape[0] if m.ndim == 3 else 1)
    out = np.empty((heads, src, dv), np.float32)
    ok = np.empty((groups, past + cur, d), np.float32) if want_cache else None
    ov = np.empty((groups, past + cur, dv), np.float32) if want_cache else None
    rc = lib().orc_sdpa(_p(q), heads, src, d, _p(k), _p(v), groups, cur, dv, _p(m), mask_c, _p(pk),
                        _p(pv), past, float(scale), _p(out), _p(ok), _p(ov))
    if rc != 0:
        raise ValueError("orc_sdpa rejected its arguments")
    return (out, ok, ov) if want_cache else out


def timestep_embedding(inp, half_dim: int = 512, scale: float = 1000.0, max_period: float = 10000.0,
                       schedule_mode: int = 0) -> np.ndarray:
    inp = _f32(inp).ravel()
    out = np.empty((inp.size, 2 * half_dim), np.float32)
    lib().orc_timestep_embedding(_p(inp), inp.size, half_dim, scale, max_period, schedule_mode, _p(out))
    return out


def decoder_mask(cur: int, past: int) -> np.ndarray:
    out = np.empty((cur, past + cur), np.float32)
    lib().orc_decoder_mask(cur, past, _p(out))
    return out


def rope_cache(head_dim: int, theta: float, original_max: int, start: int, length: int,
               short_factor=None, long_factor=None):
    sf = _f32(np.ones(head_dim // 2) if short_factor is None else short_factor)
    lf = None if long_factor is None else _f32(long_factor)
    cos = np.empty((length, head_dim), np.float32)
    sin = np.empty((length, head_dim), np.float32)
    lib().orc_rope_cache(head_dim, theta, original_max, _p(sf), _p(lf), start, length, _p(cos), _p(sin))
    return cos, sin


def sway_t_span(timesteps: int) -> np.ndarray:
    out = np.empty(timesteps + 1, np.float32)
    lib().orc_sway_t_span(timesteps, _p(out))
    return out


def zero_init_steps(timesteps: int) -> int:
    return lib().orc_zero_init_steps(timesteps)


def optimized_scale(pos, neg) -> float:
    pos, neg = _f32(pos), _f32(neg)
    return float(lib().orc_optimized_scale(_p(pos), _p(neg), pos.size))


def max_patches(target_text_tokens: int, hard_cap: int = 2000) -> int:
    return lib().orc_max_patches(target_text_tokens, hard_cap)


def noise_table(seed: int, patches: int, per_patch: int = 256) -> np.ndarray:
    out = np.empty((patches, per_patch), np.float32)
    lib().orc_noise_table(seed, patches, per_patch, _p(out))
    return out


# ------------------------------------------------------------ model ------
class Oracle:
    """The reference's ncnn CPU path for one model, restated in fp32."""

    def __init__(self, cfg: ModelConfig, blobs: Dict[int, np.ndarray]):
        self.cfg = cfg
        self._desc = desc(cfg)
        L = lib()
        self._m = L.orc_model_create(C.byref(self._desc))
        self._blobs = {}
        for comp, blob in blobs.items():
            blob = np.ascontiguousarray(blob, dtype=np.float16)
            n = L.orc_component_count(C.byref(self._desc), comp)
            if n != blob.size or n != component_count(cfg, comp):
                raise ValueError(f"component {comp}: blob has {blob.size} values, oracle expects {n}")
            self._blobs[comp] = blob
            if L.orc_set_weights(self._m, comp, _p(blob), blob.size) != 0:
                raise ValueError(f"orc_set_weights({comp}) failed")

    def __del__(self):
        m = getattr(self, "_m", None)
        if m:
            lib().orc_model_destroy(m)
            self._m = None

    def set_rope_factors(self, short_factor, long_factor=None) -> None:
        """The base decoder's LongRoPE factors (at least head_dim / 2 values each; long optional)."""
        self._sf = np.ascontiguousarray(short_factor, dtype=np.float32)
        self._lf = None if long_factor is None else np.ascontiguousarray(long_factor, dtype=np.float32)
        rc = lib().orc_set_rope_factors(self._m, _p(self._sf), _p(self._lf) if self._lf is not None else None,
                                        self._sf.size)
        if rc != 0:
            raise ValueError("rope factors: at least head_dim / 2 positive values each")

    def reset(self) -> None:
        lib().orc_reset_caches(self._m)

    def token_count(self, which: int) -> int:
        return lib().orc_token_count(self._m, which)

    def read_cache(self, which: int, layer: int):
        n = self.token_count(which)
        k = np.empty((self.cfg.kv_heads, n, self.cfg.head_dim), np.float32)
        v = np.empty_like(k)
        if lib().orc_read_cache(self._m, which, layer, _p(k), _p(v)) != 0:
            raise ValueError("bad cache index")
        return k, v

    def decoder_forward(self, which: int, embed, mask=None, cos=None, sin=None) -> np.ndarray:
        embed = _f32(embed)
        n = embed.shape[0]
        out = np.empty((n, self.cfg.hidden), np.float32)
        m = None if mask is None else _f32(mask)
        c = None if cos is None else _f32(cos)
        s = None if sin is None else _f32(sin)
        if lib().orc_decoder_forward(self._m, which, _p(embed), n, _p(m), _p(c), _p(s), _p(out)) != 0:
            raise ValueError("orc_decoder_forward failed")
        return out

    def text_embed(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.cfg.hidden), np.float32)
        if lib().orc_text_embed(self._m, _p(ids), ids.size, _p(out)) != 0:
            raise ValueError("token id out of range")
        return out

    def fsq(self, x) -> np.ndarray:
        x = _f32(x).reshape(-1, self.cfg.hidden)
        out = np.empty_like(x)
        lib().orc_fsq(self._m, _p(x), x.shape[0], _p(out))
        return out

    def fusion_proj(self, lm, feat) -> np.ndarray:
        lm = _f32(lm).reshape(-1, self.cfg.hidden)
        feat = _f32(feat).reshape(-1, self.cfg.hidden)
        out = np.empty_like(lm)
        lib().orc_fusion_proj(self._m, _p(lm), _p(feat), lm.shape[0], _p(out))
        return out

    def dit_proj(self, lm, res) -> np.ndarray:
        out = np.empty(2 * self.cfg.dit_hidden, np.float32)
        lib().orc_dit_proj(self._m, _p(_f32(lm)), _p(_f32(res)), _p(out))
        return out

    def stop_head(self, h) -> np.ndarray:
        out = np.empty(2, np.float32)
        lib().orc_stop_head(self._m, _p(_f32(h)), _p(out))
        return out

    def feat_encoder(self, latent_dp) -> np.ndarray:
        out = np.empty(self.cfg.hidden, np.float32)
        lib().orc_feat_encoder(self._m, _p(_f32(latent_dp)), _p(out))
        return out

    def dit_estimator(self, x_in, mu_in, t_in, cond_in, dt_in) -> np.ndarray:
        out = np.empty((2, self.cfg.latent), np.float32)
        rc = lib().orc_dit_estimator(self._m, _p(_f32(x_in)), _p(_f32(mu_in)), _p(_f32(t_in)),
                                     _p(_f32(cond_in)), _p(_f32(dt_in)), _p(out))
        if rc != 0:
            raise ValueError("orc_dit_estimator failed")
        return out

    def cfm_sample(self, mu, cond, noise, timesteps: int = 10, cfg_value: float = 2.0) -> np.ndarray:
        out = np.empty(self.cfg.latent, np.float32)
        rc = lib().orc_cfm_sample(self._m, _p(_f32(mu)), _p(_f32(cond)), _p(_f32(noise)), timesteps,
                                  cfg_value, _p(out))
        if rc == -2:
            raise RuntimeError("dit_estimator produced non-finite values")
        if rc != 0:
            raise ValueError("orc_cfm_sample failed")
        return out

    def generate(self, text_ids, min_patches: int = 2, timesteps: int = 10, cfg_value: float = 2.0,
                 max_patches_override: int = 0, seed: int = 0, fsq_codes=None) -> dict:
        """generate_with_caches for a text-only prefix. fsq_codes [rows][fsq_dim]: codes
        that replace the FSQ rounding of patches 0 .. rows - 1 (the test hook that lets
        the oracle follow another run's rounding decisions; see orc_force_fsq)."""
        ids = np.ascontiguousarray(text_ids, dtype=np.int32)
        cap = max_patches(ids.size, self.cfg.max_generation_patches)
        if max_patches_override > 0:
            cap = min(cap, max_patches_override)
        lat = np.zeros((cap, self.cfg.latent), np.float32)
        lm = np.zeros((cap, self.cfg.hidden), np.float32)
        res = np.zeros((cap, self.cfg.hidden), np.float32)
        stop = np.zeros((cap, 2), np.float32)
        fsq_pre = np.zeros((cap, self.cfg.fsq_dim), np.float32)
        n = C.c_int(0)
        codes = None if fsq_codes is None else np.ascontiguousarray(fsq_codes, dtype=np.float32)
        lib().orc_trace_fsq(self._m, _p(fsq_pre), cap)
        if codes is not None:
            lib().orc_force_fsq(self._m, _p(codes), codes.shape[0])
        try:
            rc = lib().orc_generate(self._m, _p(ids), ids.size, min_patches, timesteps, cfg_value,
                                    max_patches_override, seed, _p(lat), _p(lm), _p(res), _p(stop), C.byref(n))
        finally:
            lib().orc_trace_fsq(self._m, None, 0)
            lib().orc_force_fsq(self._m, None, 0)
        if rc == -2:
            raise RuntimeError("dit_estimator produced non-finite values")
        if rc == -3:
            raise RuntimeError("VoxCPM2 KV cache reached the exported RoPE range")
        if rc != 0:
            raise ValueError("orc_generate failed")
        k = n.value
        # fsq_pre[p]: the FSQ values of patch p before rounding (tanh(z) * fsq_scale); their
        # rounded codes make the LM hidden state entering patch p + 1
        return {"patches": k, "latents": lat[:k], "lm_hidden": lm[:k], "res_hidden": res[:k],
                "stop_logits": stop[:k], "fsq_pre": fsq_pre[:k]}

    def generate_rows(self, token_ids, is_audio, audio_latents, n_target_text: int, min_patches: int = 2,
                      timesteps: int = 10, cfg_value: float = 2.0, max_patches_override: int = 0,
                      seed: int = 0) -> dict:
        """generate() from a prefix given row by row: token ids, is_audio flags and
        the audio rows' latent patches ([n_audio][D*P], d-major, row order)."""
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        flags = np.ascontiguousarray(is_audio, dtype=np.int32)
        if flags.shape != ids.shape:
            raise ValueError("one is_audio flag per row")
        lat_in = None if audio_latents is None else _f32(audio_latents).reshape(-1, self.cfg.latent)
        cap = max_patches(n_target_text, self.cfg.max_generation_patches)
        if max_patches_override > 0:
            cap = min(cap, max_patches_override)
        lat = np.zeros((cap, self.cfg.latent), np.float32)
        lm = np.zeros((cap, self.cfg.hidden), np.float32)
        res = np.zeros((cap, self.cfg.hidden), np.float32)
        stop = np.zeros((cap, 2), np.float32)
        n = C.c_int(0)
        rc = lib().orc_generate_rows(self._m, _p(ids), _p(flags), _p(lat_in), ids.size, n_target_text, min_patches,
                                     timesteps, cfg_value, max_patches_override, seed, _p(lat), _p(lm), _p(res),
                                     _p(stop), C.byref(n))
        if rc == -2:
            raise RuntimeError("dit_estimator produced non-finite values")
        if rc == -3:
            raise RuntimeError("VoxCPM2 KV cache reached the exported RoPE range")
        if rc != 0:
            raise ValueError("orc_generate_rows failed")
        k = n.value
        return {"patches": k, "latents": lat[:k], "lm_hidden": lm[:k], "res_hidden": res[:k],
                "stop_logits": stop[:k]}
