"""The CPU oracle against the reference's known-answer tests and the torch restatement."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest

import oracle
from voxcpm2_b200.config import BENCH, COMPONENTS, TINY, component_count


def test_sdpa_kat(kat):
    # tests/test_voxcpm2_sdpa.cpp:121-124 checks the CPU layer at 1e-5
    out = oracle.sdpa(kat["sdpa_q"], kat["sdpa_k"], kat["sdpa_v"])
    assert np.abs(out - kat["sdpa_out"]).max() <= 1e-5


def test_timestep_embedding_kat(kat):
    # tests/test_voxcpm2_timestep_embedding.cpp:165-170: raw and schedule modes at 1e-6
    raw = oracle.timestep_embedding(kat["ts_raw_in"], 512, 1000.0, 10000.0, 0)
    assert np.abs(raw - kat["ts_raw_out"]).max() <= 1e-6
    sched = oracle.timestep_embedding(kat["ts_sched_in"], 512, 1000.0, 10000.0, 1)
    assert np.abs(sched - kat["ts_sched_out"]).max() <= 1e-6


def test_kvcache_toy_growth(kat):
    """tests/test_kvcache.cpp:80-111: two cached SDPA layers, prefill 2 then 2 decode steps."""
    caches = [(None, None), (None, None)]
    for step in range(3):
        x = kat[f"kv_in{step}"]
        n = x.shape[0]
        h = x
        for layer in range(2):
            pk, pv = caches[layer]
            past = 0 if pk is None else pk.shape[1]
            mask = oracle.decoder_mask(n, past)
            h3 = h[None]
            out, nk, nv = oracle.sdpa(h3, h3, h3, mask=mask, past_k=pk, past_v=pv, scale=0.5,
                                      want_cache=True)
            caches[layer] = (nk, nv)
            h = out[0]
        assert caches[0][0].shape[1] == kat["kv_counts"][step]
        assert np.abs(h - kat[f"kv_out{step}"]).max() <= 1e-6


def test_decoder_mask():
    m = oracle.decoder_mask(3, 2)
    assert m.shape == (3, 5)
    assert (m[0] == [0, 0, 0, -1e4, -1e4]).all()
    assert (m[2] == 0).all()
    assert (oracle.decoder_mask(1, 7) == 0).all()


def test_sway_schedule_and_zero_init(kat):
    assert np.abs(oracle.sway_t_span(10) - kat["t_span10"]).max() <= 1e-7
    assert oracle.zero_init_steps(10) == int(kat["zero_init10"][0]) == 1
    assert oracle.zero_init_steps(49) == 2  # int(50 * 0.04) = 2


def test_optimized_scale_double_accumulation():
    rng = np.random.default_rng(3)
    p, n = rng.standard_normal(256).astype(np.float32), rng.standard_normal(256).astype(np.float32)
    want = np.float32((p.astype(np.float64) @ n) / (1e-8 + n.astype(np.float64) @ n))
    assert oracle.optimized_scale(p, n) == want


def test_max_patches_rule():
    # synthesizer.cpp:216-220
    assert oracle.max_patches(64, 2000) == 394
    assert oracle.max_patches(0, 2000) == 16
    assert oracle.max_patches(1000, 2000) == 2000


def test_rope_table_half_duplicated():
    cos, sin = oracle.rope_cache(64, 10000.0, 32768, 5, 3)
    assert np.array_equal(cos[:, :32], cos[:, 32:]) and np.array_equal(sin[:, :32], sin[:, 32:])
    inv = np.float32(1.0) / np.power(np.float32(10000.0), (2.0 * np.arange(32) / 64).astype(np.float32))
    assert np.allclose(cos[1, :32], np.cos(np.float32(6.0) * inv), atol=1e-6)


def test_rope_long_factor_switch():
    # synthesizer.cpp:945-948: long factors once position_start + length > original max
    short = np.ones(32, np.float32)
    long = np.full(32, 4.0, np.float32)
    c1, _ = oracle.rope_cache(64, 10000.0, 100, 90, 10, short, long)
    c2, _ = oracle.rope_cache(64, 10000.0, 100, 90, 11, short, long)
    assert np.allclose(c1[0, :32], np.cos(90 * np.power(10000.0, -2.0 * np.arange(32) / 64)), atol=1e-5)
    assert np.allclose(c2[0, :32], np.cos(90 / 4.0 * np.power(10000.0, -2.0 * np.arange(32) / 64)), atol=1e-5)


def test_decoder_rope_factors(tiny_blobs):
    """LongRoPE factors set on the model rotate the base decoder's q/k exactly as
    the tables make_rope_cache builds for the call's range (short below original
    max, long once start + n exceeds it); the residual decoder has no RoPE."""
    cfg = dataclasses.replace(TINY, rope_original_max=12)
    rng = np.random.default_rng(3)
    short = rng.uniform(0.5, 2.0, cfg.head_dim // 2).astype(np.float32)
    long = rng.uniform(2.0, 8.0, cfg.head_dim // 2).astype(np.float32)
    x = rng.standard_normal((14, cfg.hidden), dtype=np.float32)
    plain = oracle.Oracle(cfg, tiny_blobs)
    o = oracle.Oracle(cfg, tiny_blobs)
    o.set_rope_factors(short, long)
    ref = oracle.Oracle(cfg, tiny_blobs)
    for start, n in ((0, 8), (8, 1), (9, 5)):  # the last call ends at 14 > 12: long factors
        rows = x[start:start + n]
        cos, sin = oracle.rope_cache(cfg.head_dim, cfg.rope_theta, 12, start, n, short, long)
        got = o.decoder_forward(0, rows)
        assert np.array_equal(got, ref.decoder_forward(0, rows, cos=cos, sin=sin))
        assert not np.allclose(got, plain.decoder_forward(0, rows), atol=1e-6)
    assert np.array_equal(o.decoder_forward(1, x[:3]), plain.decoder_forward(1, x[:3]))
    with pytest.raises(ValueError):
        o.set_rope_factors(short[:-1])
    with pytest.raises(ValueError):
        o.set_rope_factors(-short)


def test_noise_table_is_libstdcxx_stream():
    # Fresh normal_distribution per patch from one mt19937(0): with an even draw
    # count per patch the stream is the same as one continuous draw.
    a = oracle.noise_table(0, 3, 256)
    b = oracle.noise_table(0, 1, 768).reshape(3, 256)
    assert np.array_equal(a, b)
    assert abs(float(a.mean())) < 0.2 and 0.8 < float(a.std()) < 1.2


def test_component_counts_agree():
    for cfg in (TINY, BENCH):
        d = oracle.desc(cfg)
        for c in COMPONENTS:
            assert oracle.lib().orc_component_count(oracle.oracle.C.byref(d), c) == component_count(cfg, c)


def test_oracle_matches_torch_restatement(tiny_golden, tiny_blobs):
    g = tiny_golden
    o = oracle.Oracle(TINY, tiny_blobs)
    for which in (0, 1):
        o.reset()
        out = o.decoder_forward(which, g["pre"])
        assert np.abs(out - g[f"dec{which}_pre_out"]).max() < 2e-4
        for s in range(2):
            out = o.decoder_forward(which, g["steps"][s:s + 1])
            assert np.abs(out - g[f"dec{which}_step{s}_out"]).max() < 2e-4
        assert o.token_count(which) == 7
    est = o.dit_estimator(g["dit_x"], g["dit_mu"], g["dit_t"], g["dit_cond"], g["dit_dt"])
    assert np.abs(est - g["dit_out"]).max() < 2e-4
    assert np.abs(o.fsq(g["h"])[0] - g["fsq_out"]).max() < 2e-4
    assert np.abs(o.stop_head(g["h"]) - g["stop_out"]).max() < 1e-5
    assert np.abs(o.feat_encoder(g["lat"]) - g["feat_out"]).max() < 1e-4
    assert np.abs(o.fusion_proj(g["h"], g["h2"])[0] - g["fusion_out"]).max() < 1e-4
    assert np.abs(o.dit_proj(g["h"], g["h2"]) - g["ditproj_out"]).max() < 1e-4


def test_cfm_sample_zero_init_skips_first_step(tiny_blobs):
    o = oracle.Oracle(TINY, tiny_blobs)
    rng = np.random.default_rng(5)
    mu = rng.standard_normal(2 * TINY.dit_hidden).astype(np.float32)
    cond = rng.standard_normal(TINY.latent).astype(np.float32)
    noise = rng.standard_normal(TINY.latent).astype(np.float32)
    # T = 1: zero_init_steps = 1 -> no estimator call, the latent is the noise.
    assert np.array_equal(o.cfm_sample(mu, cond, noise, timesteps=1), noise)
    x = o.cfm_sample(mu, cond, noise, timesteps=10, cfg_value=2.0)
    assert np.isfinite(x).all() and not np.array_equal(x, noise)


def test_generate_stop_rule_and_cap(tiny_blobs):
    o = oracle.Oracle(TINY, tiny_blobs)
    ids = np.arange(1, 9, dtype=np.int32)
    r = o.generate(ids, min_patches=3, timesteps=4, max_patches_override=20)
    n = r["patches"]
    logits = r["stop_logits"]
    # no stop at or before min_patches; stop at the first later step with l1 > l0
    later = [s for s in range(4, 20) if logits[s, 1] > logits[s, 0]] if n == 20 else None
    if n < 20:
        s = n - 1
        assert s > 3 and logits[s, 1] > logits[s, 0]
        assert all(not (logits[k, 1] > logits[k, 0]) for k in range(4, s))
    else:
        assert not later


def test_generate_rows_text_prefix_matches_generate(tiny_blobs):
    """A row-by-row prefix of the target ids + audio_start, with no audio rows, is
    generate()'s prefix (synthesizer.cpp:387-390): identical results."""
    o = oracle.Oracle(TINY, tiny_blobs)
    ids = np.arange(3, 11, dtype=np.int32)
    want = o.generate(ids, min_patches=100, timesteps=4, max_patches_override=5, seed=3)
    rows = np.append(ids, TINY.audio_start_token).astype(np.int32)
    got = o.generate_rows(rows, np.zeros(rows.size, np.int32), None, ids.size, min_patches=100, timesteps=4,
                          max_patches_override=5, seed=3)
    assert got["patches"] == want["patches"]
    for k in ("latents", "lm_hidden", "res_hidden", "stop_logits"):
        assert np.array_equal(got[k], want[k]), k


def test_generate_rows_audio_prefix(tiny_blobs):
    """Audio rows change the prefix (feat_encoder embeddings, FSQ'd LM rows, the
    residual decoder's feature input) and, when last, condition the first patch."""
    o = oracle.Oracle(TINY, tiny_blobs)
    ids = np.arange(3, 9, dtype=np.int32)
    rng = np.random.default_rng(5)
    audio = rng.standard_normal((3, TINY.latent)).astype(np.float32)
    rows = np.concatenate([ids, [TINY.audio_start_token, 0, 0, 0]]).astype(np.int32)
    flags = np.array([0] * (ids.size + 1) + [1, 1, 1], np.int32)
    a = o.generate_rows(rows, flags, audio, ids.size, min_patches=100, timesteps=4, max_patches_override=4, seed=1)
    text = o.generate_rows(rows[:ids.size + 1], flags[:ids.size + 1], None, ids.size, min_patches=100, timesteps=4,
                           max_patches_override=4, seed=1)
    assert a["patches"] == text["patches"] == 4
    assert np.all(np.isfinite(a["latents"]))
    assert not np.allclose(a["latents"], text["latents"])
    assert not np.allclose(a["lm_hidden"][0], text["lm_hidden"][0])
    with pytest.raises(ValueError):
        o.generate_rows(rows, flags, None, ids.size, max_patches_override=2)  # audio rows without latents


def test_fsq_trace_and_forced_codes_reproduce_the_loop():
    """The FSQ test hooks: the codes recovered from the traced LM hidden states are
    the oracle's own rounding of its traced pre-rounding values, and forcing those
    codes back reproduces the loop bit for bit; forcing one other code changes the
    patches after it."""
    from conftest import fsq_codes_from_hidden, fsq_forced_disagreements
    from voxcpm2_b200 import synthetic
    blobs = synthetic.model_blobs(TINY, 0)
    orc = oracle.Oracle(TINY, blobs)
    ids = synthetic.token_ids(TINY, 8, seed=3)
    a = orc.generate(ids, min_patches=100, timesteps=4, cfg_value=2.0, max_patches_override=8, seed=1)
    codes, resid = fsq_codes_from_hidden(TINY, blobs, a["lm_hidden"][1:])
    assert resid < 1e-3
    assert np.array_equal(codes, np.rint(a["fsq_pre"][:7]))
    b = orc.generate(ids, min_patches=100, timesteps=4, cfg_value=2.0, max_patches_override=8, seed=1, fsq_codes=codes)
    assert np.array_equal(a["latents"], b["latents"]) and np.array_equal(a["lm_hidden"], b["lm_hidden"])
    assert fsq_forced_disagreements(b["fsq_pre"], codes) == []
    other = codes[:3].copy()  # patches 3 on round their own values
    other[2, 5] += 1.0
    c = orc.generate(ids, min_patches=100, timesteps=4, cfg_value=2.0, max_patches_override=8, seed=1, fsq_codes=other)
    # the FSQ of patch 2 makes the LM state entering patch 3
    assert np.array_equal(a["latents"][:3], c["latents"][:3]) and not np.array_equal(a["latents"][3], c["latents"][3])
    d = fsq_forced_disagreements(c["fsq_pre"], other)
    assert len(d) == 1 and d[0][:4] == (2, 5, codes[2, 5], codes[2, 5] + 1.0)
