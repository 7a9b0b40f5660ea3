"""Generate the golden fixtures under tests/golden/ (run: python tests/golden/make_golden.py).

kat.npz -- the reference's own known-answer tests, restated in numpy fp32:
  * SDPA (tests/test_voxcpm2_sdpa.cpp:24-30 inputs, :82-114 closed-form reference):
    q [2 heads][2][4] = sin(0.17 i + 0.1), k/v [1 group][2][4] with offsets 0.2/0.3,
    no mask, scale 1/sqrt(4); the test's tolerance is 1e-5.
  * timestep embedding (tests/test_voxcpm2_timestep_embedding.cpp:110-160): half_dim 512,
    scale 1000, period 1e4; raw t = {0.70710677, 0.25} and schedule (1, 10); tolerance 1e-6.
  * KV-cache toy decoder (tests/test_kvcache.cpp:22-111): two SDPA layers (5=1 6=0.5 7=1),
    head_dim 4, one KV head, q=k=v=input; prefill 2 tokens then 2 decode steps with the
    causal -1e4 mask of make_decoder_mask; token counts 2 -> 3 -> 4.
  * sway schedule t_span (synthesizer.cpp:55-59) and zero-init steps (:123) for T = 10.

tiny_model.npz -- the exporter's graphs (tools/export_components.py:496-689) run by the
torch restatement in tests/torch_ref.py on the TINY config's seed-0 synthetic weights.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

OUT = Path(__file__).resolve().parent
f32 = np.float32


def values(count, offset):
    i = np.arange(count, dtype=f32)
    return np.sin(i * f32(0.17) + f32(offset)).astype(f32)


def sdpa_kat():
    q = values(16, 0.1).reshape(2, 2, 4)
    k = values(8, 0.2).reshape(1, 2, 4)
    v = values(8, 0.3).reshape(1, 2, 4)
    scale = f32(1.0) / f32(math.sqrt(4.0))
    out = np.zeros((2, 2, 4), f32)
    for h in range(2):
        for i in range(2):
            s = np.array([np.sum(q[h, i] * k[0, j], dtype=f32) * scale for j in range(2)], f32)
            s = np.exp(s - s.max()).astype(f32)
            s = (s / s.sum()).astype(f32)
            out[h, i] = s[0] * v[0, 0] + s[1] * v[0, 1]
    return q, k, v, out


def timestep_reference(ts):
    out = np.zeros((2, 1024), f32)
    log_period = f32(math.log(10000.0))
    for b in range(2):
        t = f32(ts[b]) * f32(1000.0)
        for i in range(512):
            # float arithmetic as in the test: std::exp(-log_period * float(i) / 511.0f)
            arg = f32(f32(-log_period * f32(i)) / f32(511.0))
            inv = f32(math.exp(float(arg)))
            ph = f32(t * inv)
            out[b, i] = math.sin(ph)
            out[b, 512 + i] = math.cos(ph)
    return out


def schedule_t(step, timesteps):
    u = f32(1.0) - f32(step) / f32(timesteps)
    return f32(u + (f32(math.cos(f32(math.pi) * f32(0.5) * u)) - f32(1.0) + u))


def toy_sdpa(x, cache, scale=0.5):
    """One Split->SDPA layer of the kvcache toy: q=k=v=x [n][4], cache [past][4]."""
    n = x.shape[0]
    past = cache.shape[0]
    kv = np.concatenate([cache, x], 0)
    mask = np.zeros((n, past + n), f32)
    for r in range(n):
        mask[r, past + r + 1:] = -10000.0
    s = (x @ kv.T).astype(f32) * f32(scale) + mask
    s = np.exp(s - s.max(1, keepdims=True)).astype(f32)
    s = s / s.sum(1, keepdims=True)
    return (s @ kv).astype(f32), kv


def make_embed(tokens, offset):
    return (f32(offset) + (np.arange(4 * tokens, dtype=f32) + 1) * f32(0.125)).reshape(tokens, 4)


def kvcache_toy():
    caches = [np.zeros((0, 4), f32), np.zeros((0, 4), f32)]
    inputs, outputs, counts = [], [], []
    for step, (tokens, off) in enumerate([(2, 0.0), (1, 1.0), (1, 2.0)]):
        x = make_embed(tokens, off)
        inputs.append(x)
        h = x
        for layer in range(2):
            h, caches[layer] = toy_sdpa(h, caches[layer])
        outputs.append(h)
        counts.append(caches[0].shape[0])
    return inputs, outputs, counts


def main():
    q, k, v, out = sdpa_kat()
    raw = np.array([0.70710677, 0.25], f32)
    sched = schedule_t(1.0, 10.0)
    t_in, t_out, counts = kvcache_toy()
    t_span = np.array([schedule_t(i, 10) for i in range(11)], f32)
    np.savez(
        OUT / "kat.npz",
        sdpa_q=q, sdpa_k=k, sdpa_v=v, sdpa_out=out,
        ts_raw_in=raw, ts_raw_out=timestep_reference(raw),
        ts_sched_in=np.array([1.0, 10.0], f32), ts_sched_out=timestep_reference([sched, sched]),
        kv_in0=t_in[0], kv_in1=t_in[1], kv_in2=t_in[2],
        kv_out0=t_out[0], kv_out1=t_out[1], kv_out2=t_out[2], kv_counts=np.array(counts, np.int32),
        t_span10=t_span, zero_init10=np.array([max(1, int((10 + 1) * 0.04))], np.int32),
    )

    import torch
    from torch_ref import TorchModel
    from voxcpm2_b200 import synthetic
    from voxcpm2_b200.config import TINY

    cfg = TINY
    blobs = synthetic.model_blobs(cfg, 0)
    tm = TorchModel(cfg, blobs)
    rng = np.random.default_rng(7)
    pre = rng.standard_normal((5, cfg.hidden)).astype(f32)
    steps = rng.standard_normal((2, cfg.hidden)).astype(f32)
    fx = {"pre": pre, "steps": steps}
    with torch.no_grad():
        for which in (0, 1):
            tm.reset()
            fx[f"dec{which}_pre_out"] = tm.decoder(which, pre).numpy()
            for s in range(2):
                fx[f"dec{which}_step{s}_out"] = tm.decoder(which, steps[s:s + 1]).numpy()
        x = rng.standard_normal((2, cfg.latent)).astype(f32)
        x[1] = x[0]
        mu = np.zeros((2, 2 * cfg.dit_hidden), f32)
        mu[0] = rng.standard_normal(2 * cfg.dit_hidden).astype(f32)
        cond = np.tile(rng.standard_normal(cfg.latent).astype(f32), (2, 1))
        t_in = np.array([3.0, 10.0], f32)
        dt = np.zeros(2, f32)
        fx.update(dit_x=x, dit_mu=mu, dit_cond=cond, dit_t=t_in, dit_dt=dt,
                  dit_out=tm.dit(x, mu, t_in, cond, dt).numpy())
        h = rng.standard_normal(cfg.hidden).astype(f32)
        h2 = rng.standard_normal(cfg.hidden).astype(f32)
        lat = rng.standard_normal(cfg.latent).astype(f32)
        fx.update(h=h, h2=h2, lat=lat,
                  fsq_out=tm.fsq(h).numpy(), stop_out=tm.stop_head(h).numpy(),
                  feat_out=tm.feat_encoder(lat).numpy(), fusion_out=tm.fusion_proj(h, h2).numpy(),
                  ditproj_out=tm.dit_proj(h, h2).numpy())
    np.savez(OUT / "tiny_model.npz", **fx)
    print("wrote", OUT / "kat.npz", OUT / "tiny_model.npz")


if __name__ == "__main__":
    main()
