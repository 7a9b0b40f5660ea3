"""Torch-CPU restatement of the exporter's component graphs (cross-check of the oracle).

tools/export_components.py defines what each ncnn graph computes:
``DecoderKv.forward`` (:496-550), ``DitEstimator.forward`` (:602-689) and the small
graphs (:553-599). This module re-runs those definitions with torch fp32
operators (``F.scaled_dot_product_attention`` with ``enable_gqa``), on the same
fp16 weights, so the C++ oracle is checked by an independent implementation.
The upstream layers the exporter calls (RMSNorm, SwiGLU ``mlp``,
``apply_rotary_pos_emb``) are written out from their published definitions.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from voxcpm2_b200.config import ModelConfig, component_offsets


class Weights:
    def __init__(self, cfg: ModelConfig, comp: int, blob: np.ndarray):
        self.t = {}
        flat = torch.from_numpy(np.asarray(blob, dtype=np.float16).astype(np.float32))
        for name, (off, shape) in component_offsets(cfg, comp).items():
            n = int(np.prod(shape))
            self.t[name] = flat[off:off + n].reshape(shape)

    def __getitem__(self, k):
        return self.t[k]


def rmsnorm(x, g, eps):
    var = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * g


def rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(q, k, cos, sin):
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def rope_table(head_dim, theta, start, length):
    half = head_dim // 2
    inv = np.array([1.0 / np.power(np.float32(theta), np.float32(2.0 * j / head_dim), dtype=np.float32)
                    for j in range(half)], dtype=np.float32)
    pos = np.arange(start, start + length, dtype=np.float32)
    freq = (pos[:, None] / np.float32(1.0)) * inv[None, :]
    cos = np.cos(freq).astype(np.float32)
    sin = np.sin(freq).astype(np.float32)
    return torch.from_numpy(np.concatenate([cos, cos], 1)), torch.from_numpy(np.concatenate([sin, sin], 1))


def causal_mask(cur, past):
    m = torch.zeros(cur, past + cur)
    for r in range(cur):
        m[r, past + r + 1:] = -10000.0
    return m


def decoder_layers(w: Weights, prefix: str, layers: int, hidden, hq, hkv, hd, eps, rscale,
                   rope=None, mask=None, cache=None):
    """DecoderKv.forward / DitEstimator.decoder body. cache: list of (k, v) [1][hkv][T][hd] or None."""
    bsz, n, _ = hidden.shape
    new_cache = []
    for i in range(layers):
        p = f"{prefix}layers.{i}."
        residual = hidden
        normed = rmsnorm(hidden, w[p + "input_layernorm"], eps)
        q = (normed @ w[p + "q_proj"].T).view(bsz, n, hq, hd).transpose(1, 2)
        k = (normed @ w[p + "k_proj"].T).view(bsz, n, hkv, hd).transpose(1, 2)
        v = (normed @ w[p + "v_proj"].T).view(bsz, n, hkv, hd).transpose(1, 2)
        if rope is not None:
            q, k = apply_rope(q, k, *rope)
        if cache is not None:
            pk, pv = cache[i]
            k = torch.cat([pk, k], 2)
            v = torch.cat([pv, v], 2)
            new_cache.append((k, v))
        attn = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, enable_gqa=True)
        attn = attn.transpose(1, 2).reshape(bsz, n, hq * hd) @ w[p + "o_proj"].T
        hidden = residual + attn * rscale
        residual = hidden
        h2 = rmsnorm(hidden, w[p + "post_attention_layernorm"], eps)
        h2 = (F.silu(h2 @ w[p + "gate_proj"].T) * (h2 @ w[p + "up_proj"].T)) @ w[p + "down_proj"].T
        hidden = residual + h2 * rscale
    return rmsnorm(hidden, w[prefix + "norm"], eps), new_cache


def timestep_embedding(t, half_dim):
    freq = torch.exp(torch.arange(half_dim, dtype=torch.float32) * (-math.log(10000) / (half_dim - 1)))
    emb = 1000.0 * t.reshape(-1, 1) * freq.reshape(1, -1)
    return torch.cat((emb.sin(), emb.cos()), dim=-1)


def sway(step_index, timesteps):
    u = 1.0 - step_index / timesteps
    return u + (math.cos(math.pi * 0.5 * u) - 1.0 + u)


def dit_estimator(cfg: ModelConfig, w: Weights, x, mu, t_in, cond, dt):
    """DitEstimator.forward with the fused timestep layer's schedule mode for t."""
    Hd, hq, hkv, hd = cfg.dit_hidden, cfg.dit_q_heads, cfg.dit_kv_heads, cfg.dit_head_dim
    x = torch.as_tensor(x).reshape(2, cfg.feat_dim, cfg.patch_size)
    cond = torch.as_tensor(cond).reshape(2, cfg.feat_dim, cfg.patch_size)
    mu = torch.as_tensor(mu).reshape(2, 2 * Hd)
    xh = x.transpose(1, 2) @ w["in_proj.weight"].T + w["in_proj.bias"]
    ch = cond.transpose(1, 2) @ w["cond_proj.weight"].T + w["cond_proj.bias"]
    ts = torch.full((2,), sway(float(t_in[0]), float(t_in[1])), dtype=torch.float32)

    def mlp(name, e):
        h = F.silu(e @ w[f"{name}.linear_1.weight"].T + w[f"{name}.linear_1.bias"])
        return h @ w[f"{name}.linear_2.weight"].T + w[f"{name}.linear_2.bias"]

    tt = mlp("time_mlp", timestep_embedding(ts, Hd // 2)) + \
        mlp("delta_time_mlp", timestep_embedding(torch.as_tensor(dt, dtype=torch.float32), Hd // 2))
    mu4 = mu.reshape(-1, Hd)
    rope = rope_table(hd, cfg.rope_theta, 0, 3 + 2 * cfg.patch_size)
    outs = []
    for b in range(2):
        seq = torch.cat([mu4[2 * b:2 * b + 2], tt[b:b + 1], ch[b], xh[b]], 0)[None]
        h, _ = decoder_layers(w, "decoder.", cfg.dit_layers, seq, hq, hkv, hd, cfg.rms_eps,
                              cfg.dit_residual_scale, rope=rope)
        outs.append(h[0, 3 + cfg.patch_size:])
    hidden = torch.cat(outs, 0)
    out = (hidden @ w["out_proj.weight"].T + w["out_proj.bias"]).reshape(2, cfg.patch_size, -1)
    return out.transpose(1, 2).reshape(2, -1)


class TorchModel:
    def __init__(self, cfg: ModelConfig, blobs):
        self.cfg = cfg
        self.w = {c: Weights(cfg, c, b) for c, b in blobs.items()}
        self.cache = {0: None, 1: None}

    def reset(self):
        self.cache = {0: None, 1: None}

    def decoder(self, which, embed):
        cfg = self.cfg
        embed = torch.as_tensor(embed, dtype=torch.float32)
        n = embed.shape[0]
        layers = cfg.base_layers if which == 0 else cfg.res_layers
        if self.cache[which] is None:
            empty = torch.zeros(1, cfg.kv_heads, 0, cfg.head_dim)
            self.cache[which] = [(empty, empty)] * layers
        past = self.cache[which][0][0].shape[2]
        rope = rope_table(cfg.head_dim, cfg.rope_theta, past, n) if which == 0 else None
        rscale = cfg.base_residual_scale if which == 0 else cfg.res_residual_scale
        out, self.cache[which] = decoder_layers(
            self.w[1 + which], "", layers, embed[None], cfg.q_heads, cfg.kv_heads, cfg.head_dim,
            cfg.rms_eps, rscale, rope=rope, mask=causal_mask(n, past), cache=self.cache[which])
        return out[0]

    def dit(self, x, mu, t_in, cond, dt):
        return dit_estimator(self.cfg, self.w[8], x, mu, t_in, cond, dt)

    def fsq(self, h):
        w = self.w[3]
        z = torch.tanh(torch.as_tensor(h) @ w["in_proj.weight"].T + w["in_proj.bias"])
        z = torch.round(z * self.cfg.fsq_scale) / self.cfg.fsq_scale
        return z @ w["out_proj.weight"].T + w["out_proj.bias"]

    def stop_head(self, h):
        w = self.w[6]
        mid = F.silu(torch.as_tensor(h) @ w["stop_proj.weight"].T + w["stop_proj.bias"])
        return mid @ w["stop_head.weight"].T

    def feat_encoder(self, latent_dp):
        w = self.w[7]
        frames = torch.as_tensor(latent_dp).reshape(self.cfg.feat_dim, self.cfg.patch_size).T.reshape(-1)
        mid = F.silu(frames @ w["in_proj.weight"].T + w["in_proj.bias"])
        return mid @ w["enc_to_lm_proj.weight"].T + w["enc_to_lm_proj.bias"]

    def fusion_proj(self, lm, feat):
        w = self.w[4]
        return torch.cat([torch.as_tensor(lm), torch.as_tensor(feat)], -1) @ w["weight"].T + w["bias"]

    def dit_proj(self, lm, res):
        w = self.w[5]
        a = torch.as_tensor(lm) @ w["lm_proj.weight"].T + w["lm_proj.bias"]
        b = torch.as_tensor(res) @ w["res_proj.weight"].T + w["res_proj.bias"]
        return torch.cat([a, b], -1)
