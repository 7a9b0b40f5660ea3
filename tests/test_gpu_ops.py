"""GPU parity of the single operators against the CPU oracle, through the C ABI.

Each test runs the CUDA library on a B200 and the oracle (the reference's ncnn
CPU path restated) on the same seeded inputs and fp16 weights.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest

import oracle
from conftest import assert_parity, close_stats
from voxcpm2_b200 import synthetic
from voxcpm2_b200.config import BENCH, SMALL, TINY

pytestmark = pytest.mark.gpu

CONFIGS = {"tiny": TINY, "small": SMALL, "bench": BENCH}


@pytest.fixture(scope="module")
def rt():
    from voxcpm2_b200 import runtime
    return runtime


@pytest.fixture(scope="module")
def models(rt):
    """name -> (cfg, blobs, Device, Oracle), built lazily."""
    cache = {}

    def get(name):
        if name not in cache:
            cfg = CONFIGS[name]
            blobs = synthetic.model_blobs(cfg, 0)
            cache[name] = (cfg, blobs, rt.Device(cfg, 0, blobs), oracle.Oracle(cfg, blobs))
        return cache[name]

    yield get
    for cfg, blobs, dev, orc in cache.values():
        dev.close()


# ------------------------------------------------------------------ SDPA ---
def test_sdpa_known_answer(rt, kat):
    # tests/test_voxcpm2_sdpa.cpp:121-124 bar: 1e-5
    out = rt.sdpa(kat["sdpa_q"], kat["sdpa_k"], kat["sdpa_v"])
    assert np.abs(out - kat["sdpa_out"]).max() <= 1e-5


def test_sdpa_decode_shape_with_cache(rt):
    """One query row, 16 heads over a 512-token GQA 8:1 cache (+1 new token), scale 1/8."""
    rng = np.random.default_rng(11)
    q = rng.standard_normal((16, 1, 64), dtype=np.float32)
    pk = rng.standard_normal((2, 512, 64), dtype=np.float32)
    pv = rng.standard_normal((2, 512, 64), dtype=np.float32)
    k = rng.standard_normal((2, 1, 64), dtype=np.float32)
    v = rng.standard_normal((2, 1, 64), dtype=np.float32)
    mask = oracle.decoder_mask(1, 512)
    want, wk, wv = oracle.sdpa(q, k, v, mask, pk, pv, 0.125, want_cache=True)
    got, gk, gv = rt.sdpa(q, k, v, mask, pk, pv, 0.125, want_cache=True)
    assert np.abs(got - want).max() <= 1e-5
    assert np.array_equal(gk, wk) and np.array_equal(gv, wv)


@pytest.mark.parametrize("past,src,per_head", [(0, 3, False), (7, 5, False), (4, 2, True), (0, 1, False)])
def test_sdpa_rows_masked(rt, past, src, per_head):
    rng = np.random.default_rng(100 + past + src)
    heads, groups, d = 4, 2, 32
    q = rng.standard_normal((heads, src, d), dtype=np.float32)
    k = rng.standard_normal((groups, src, d), dtype=np.float32)
    v = rng.standard_normal((groups, src, d), dtype=np.float32)
    pk = rng.standard_normal((groups, past, d), dtype=np.float32) if past else None
    pv = rng.standard_normal((groups, past, d), dtype=np.float32) if past else None
    mask = oracle.decoder_mask(src, past)
    if per_head:
        mask = np.stack([mask + rng.standard_normal(mask.shape).astype(np.float32) * 0.1 for _ in range(heads)])
    want = oracle.sdpa(q, k, v, mask, pk, pv, 0.0)
    got = rt.sdpa(q, k, v, mask, pk, pv, 0.0)
    assert np.abs(got - want).max() <= 1e-5


@pytest.mark.parametrize("G", [1, 3, 5, 16])
@pytest.mark.parametrize("past", [700, 1500])
@pytest.mark.parametrize("masked", [False, True])
def test_sdpa_split_path_head_groups(rt, G, past, masked):
    """One query row over more than 512 keys takes the split-K flash decode, whose
    CTAs spread a KV group's G query heads over four thread groups: G = 1 and 3
    leave thread groups without a head, 5 and 16 give them uneven counts. Held to
    the oracle at the reference test's 1e-5, with and without an additive mask."""
    rng = np.random.default_rng(1000 * G + past + masked)
    groups, d = 2, 64
    heads = G * groups
    q = rng.standard_normal((heads, 1, d), dtype=np.float32)
    k = rng.standard_normal((groups, 1, d), dtype=np.float32)
    v = rng.standard_normal((groups, 1, d), dtype=np.float32)
    pk = rng.standard_normal((groups, past, d), dtype=np.float32)
    pv = rng.standard_normal((groups, past, d), dtype=np.float32)
    mask = (rng.standard_normal((1, past + 1)) * 2.0).astype(np.float32) if masked else None
    want, wk, wv = oracle.sdpa(q, k, v, mask, pk, pv, 0.125, want_cache=True)
    got, gk, gv = rt.sdpa(q, k, v, mask, pk, pv, 0.125, want_cache=True)
    assert np.abs(got - want).max() <= 1e-5
    assert np.array_equal(gk, wk) and np.array_equal(gv, wv)


@pytest.mark.parametrize("keys", [1, 7, 64, 65, 300, 512])
@pytest.mark.parametrize("G", [1, 8, 16])
def test_sdpa_single_query_op(rt, keys, G):
    """One query row over at most 512 keys (the layer's decode shape, config 1 at 512):
    the load-all-first cluster kernel, [past | cur] rows, with and without a mask,
    against the oracle at 1e-5."""
    rng = np.random.default_rng(7 * keys + G)
    groups, d = 2, 64
    heads = G * groups
    past, cur = keys - 1, 1
    q = rng.standard_normal((heads, 1, d), dtype=np.float32)
    k = rng.standard_normal((groups, cur, d), dtype=np.float32)
    v = rng.standard_normal((groups, cur, d), dtype=np.float32)
    pk = rng.standard_normal((groups, past, d), dtype=np.float32) if past else None
    pv = rng.standard_normal((groups, past, d), dtype=np.float32) if past else None
    for mask in (None, (rng.standard_normal((1, keys)) * 2.0).astype(np.float32)):
        want = oracle.sdpa(q, k, v, mask, pk, pv, 0.125)
        got = rt.sdpa(q, k, v, mask, pk, pv, 0.125)
        assert np.abs(got - want).max() <= 1e-5, (keys, G, mask is not None)


def test_timestep_embedding_known_answer(rt, kat):
    """tests/test_voxcpm2_timestep_embedding.cpp:165-170: the layer's raw mode on
    t = {0.70710677, 0.25} and schedule mode on (step 1, 10 timesteps), both at 1e-6
    (half_dim 512, scale 1000, max_period 10000)."""
    raw = rt.timestep_embedding(kat["ts_raw_in"], 512, 1000.0, 10000.0, 0)
    assert raw.shape == kat["ts_raw_out"].shape
    assert np.abs(raw - kat["ts_raw_out"]).max() <= 1e-6
    sched = rt.timestep_embedding(kat["ts_sched_in"], 512, 1000.0, 10000.0, 1)
    assert np.abs(sched - kat["ts_sched_out"]).max() <= 1e-6
    # every step of a 10-step schedule, against the oracle
    for step in range(10):
        inp = np.array([step, 10], np.float32)
        want = oracle.timestep_embedding(inp, 512, 1000.0, 10000.0, 1)
        assert np.abs(rt.timestep_embedding(inp, 512, 1000.0, 10000.0, 1) - want).max() <= 1e-6, step


def test_kvcache_toy_decoder(rt, kat):
    """tests/test_kvcache.cpp: two cached SDPA layers, prefill 2 then 2 decode steps."""
    caches = [(None, None), (None, None)]
    for step in range(3):
        h = kat[f"kv_in{step}"]
        n = h.shape[0]
        for layer in range(2):
            pk, pv = caches[layer]
            past = 0 if pk is None else pk.shape[1]
            h3 = h[None]
            out, nk, nv = rt.sdpa(h3, h3, h3, oracle.decoder_mask(n, past), pk, pv, 0.5, want_cache=True)
            caches[layer] = (nk, nv)
            h = out[0]
        assert caches[0][0].shape[1] == kat["kv_counts"][step]
        assert np.abs(h - kat[f"kv_out{step}"]).max() <= 1e-5


def test_sdpa_rejects_bad_shapes(rt):
    with pytest.raises(rt.VxcError) as e:
        rt.sdpa(np.zeros((3, 1, 8), np.float32), np.zeros((2, 1, 8), np.float32), np.zeros((2, 1, 8), np.float32))
    assert e.value.status == 1


# --------------------------------------------------------------- decoders ---
@pytest.mark.parametrize("name", ["tiny", "small", "bench"])
@pytest.mark.parametrize("which", [0, 1])
def test_decoder_prefill_then_decode(rt, models, name, which):
    cfg, blobs, dev, orc = models(name)
    s = rt.Stream(dev, kv_capacity=64)
    rng = np.random.default_rng(7 + which)
    pre = rng.standard_normal((9, cfg.hidden), dtype=np.float32)
    orc.reset()
    want = orc.decoder_forward(which, pre)
    got = s.decoder_step(which, pre)
    assert_parity(got, want, 2e-2, 0.999, f"{name} prefill")
    assert s.token_count(which) == orc.token_count(which) == 9
    for step in range(4):
        x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
        want = orc.decoder_forward(which, x)
        got = s.decoder_step(which, x)
        err, cos = assert_parity(got, want, 2e-2, 0.999, f"{name} decode step {step}")
        assert s.token_count(which) == 10 + step
    # the fp32 KV cache holds the same rows as the oracle's HostDecoderKvCache
    for layer in (0, (cfg.base_layers if which == 0 else cfg.res_layers) - 1):
        gk, gv = s.read_cache(which, layer)
        wk, wv = orc.read_cache(which, layer)
        assert gk.shape == wk.shape == (cfg.kv_heads, 13, cfg.head_dim)
        assert np.abs(gk - wk).max() <= 1e-4 * max(1.0, np.abs(wk).max())
        assert np.abs(gv - wv).max() <= 1e-4 * max(1.0, np.abs(wv).max())
    s.close()


@pytest.mark.parametrize("which", [0, 1])
def test_decoder_steps_bulk_copy_gemv(rt, models, which, monkeypatch):
    """A lone stream's decoder GEMVs in the bulk-copy form (VXC_BULK_GEMV=1: weight rows
    into shared memory before the dependency wait, one member slot) against the oracle."""
    monkeypatch.setenv("VXC_BULK_GEMV", "1")
    cfg, blobs, dev, orc = models("bench")
    s = rt.Stream(dev, kv_capacity=64)
    rng = np.random.default_rng(57 + which)
    pre = rng.standard_normal((9, cfg.hidden), dtype=np.float32)
    orc.reset()
    assert_parity(s.decoder_step(which, pre), orc.decoder_forward(which, pre), 2e-2, 0.999, "bulk prefill")
    for step in range(3):
        x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
        assert_parity(s.decoder_step(which, x), orc.decoder_forward(which, x), 2e-2, 0.999, f"bulk step {step}")
    s.close()


@pytest.mark.parametrize("name,which", [("small", 0), ("small", 1)])
def test_decoder_decode_past_512_keys(rt, models, name, which):
    """One-row steps over 900-1000 cached keys: the decode attention's CTAs walk
    several 32-key tiles each (the double-buffered path), against the oracle."""
    cfg, blobs, dev, orc = models(name)
    s = rt.Stream(dev, kv_capacity=1100)
    rng = np.random.default_rng(31 + which)
    pre = rng.standard_normal((900, cfg.hidden), dtype=np.float32) * 0.5
    orc.reset()
    orc.decoder_forward(which, pre)
    s.decoder_step(which, pre)
    for step in range(3):
        x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
        want = orc.decoder_forward(which, x)
        got = s.decoder_step(which, x)
        assert_parity(got, want, 2e-2, 0.999, f"{name} decode step {step} over {901 + step} keys")
    # and a jump to 1000 keys
    grow = rng.standard_normal((96, cfg.hidden), dtype=np.float32) * 0.5
    orc.decoder_forward(which, grow)
    s.decoder_step(which, grow)
    x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
    assert_parity(s.decoder_step(which, x), orc.decoder_forward(which, x), 2e-2, 0.999, f"{name} step at 1000 keys")
    assert s.token_count(which) == 1000
    s.close()


@pytest.mark.parametrize("name,which,n", [("tiny", 0, 128), ("tiny", 1, 129), ("small", 0, 200), ("bench", 0, 200)])
def test_decoder_prefill_row_blocks(rt, models, name, which, n):
    """Prefill longer than one 128-row block of the tensor-core linears (full block,
    one row over, and a ragged second block), then one decode step."""
    cfg, blobs, dev, orc = models(name)
    s = rt.Stream(dev, kv_capacity=256)
    rng = np.random.default_rng(11 + n)
    pre = rng.standard_normal((n, cfg.hidden), dtype=np.float32)
    orc.reset()
    want = orc.decoder_forward(which, pre)
    got = s.decoder_step(which, pre)
    assert_parity(got, want, 2e-2, 0.999, f"{name} prefill of {n} rows")
    x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
    assert_parity(s.decoder_step(which, x), orc.decoder_forward(which, x), 2e-2, 0.999, f"{name} decode after {n}")
    gk, _ = s.read_cache(which, 0)
    wk, _ = orc.read_cache(which, 0)
    assert gk.shape == wk.shape == (cfg.kv_heads, n + 1, cfg.head_dim)
    assert np.abs(gk - wk).max() <= 1e-4 * max(1.0, np.abs(wk).max())
    s.close()


def test_decoder_rope_factors(rt):
    """vxc_set_rope_factors against the oracle on both sides of original_max (24
    here): one-row steps at positions below it rotate with the short factors, at or
    past it with the long ones, and a prefill whose range passes it rotates every
    row with the long ones (make_rope_cache's rule). The rotated keys in the KV
    cache are held to 1e-4. Factors set after a stream exists apply from its next call."""
    cfg = dataclasses.replace(TINY, rope_original_max=24)
    blobs = synthetic.model_blobs(cfg, 0)
    dev = rt.Device(cfg, 0, blobs)
    s = rt.Stream(dev, kv_capacity=64)  # built before the factors are set
    rng = np.random.default_rng(5)
    short = rng.uniform(0.5, 2.0, cfg.head_dim // 2).astype(np.float32)
    long = rng.uniform(2.0, 8.0, cfg.head_dim // 2).astype(np.float32)
    dev.set_rope_factors(short, long)
    orc = oracle.Oracle(cfg, blobs)
    orc.set_rope_factors(short, long)
    x = rng.standard_normal((30, cfg.hidden), dtype=np.float32)
    assert_parity(s.decoder_step(0, x[:10]), orc.decoder_forward(0, x[:10]), 2e-2, 0.999, "prefill of 10")
    for p in range(10, 30):
        assert_parity(s.decoder_step(0, x[p:p + 1]), orc.decoder_forward(0, x[p:p + 1]), 2e-2, 0.999,
                      f"step at position {p}")

    def same_keys(st, what):
        for layer in (0, cfg.base_layers - 1):
            gk, _ = st.read_cache(0, layer)
            wk, _ = orc.read_cache(0, layer)
            assert gk.shape == wk.shape, what
            assert np.abs(gk - wk).max() <= 1e-4 * max(1.0, np.abs(wk).max()), f"{what}, layer {layer}"

    same_keys(s, "steps across original_max")
    s2 = rt.Stream(dev, kv_capacity=64)
    orc.reset()
    assert_parity(s2.decoder_step(0, x), orc.decoder_forward(0, x), 2e-2, 0.999, "prefill of 30 (long factors)")
    same_keys(s2, "prefill past original_max")
    with pytest.raises(rt.VxcError):
        dev.set_rope_factors(short[:-1])
    with pytest.raises(rt.VxcError):
        dev.set_rope_factors(-short)
    s.close()
    s2.close()
    dev.close()


def test_decoder_capacity_checked_before_launch(rt, models):
    cfg, blobs, dev, orc = models("tiny")
    s = rt.Stream(dev, kv_capacity=4)
    s.decoder_step(0, np.zeros((3, cfg.hidden), np.float32))
    with pytest.raises(rt.VxcError) as e:
        s.decoder_step(0, np.zeros((2, cfg.hidden), np.float32))
    assert e.value.status == 1
    assert s.token_count(0) == 3  # the failed call left the cache untouched
    s.decoder_step(0, np.zeros((1, cfg.hidden), np.float32))
    assert s.token_count(0) == 4
    s.close()


# ------------------------------------------------------------ small graphs ---
@pytest.mark.parametrize("name", ["tiny", "bench"])
def test_small_graphs(rt, models, name):
    cfg, blobs, dev, orc = models(name)
    s = rt.Stream(dev, kv_capacity=16)
    rng = np.random.default_rng(3)
    h = rng.standard_normal(cfg.hidden, dtype=np.float32)
    h2 = rng.standard_normal(cfg.hidden, dtype=np.float32)
    lat = rng.standard_normal(cfg.latent, dtype=np.float32)
    # fsq rounds tanh(x) * 9: an input within float noise of a rounding boundary may
    # land on the neighbouring level; the bar still holds (one level moves <= 0.02 / 9 * |w|)
    assert_parity(s.run_component(3, h), orc.fsq(h)[0], 2e-2, 0.999, "fsq")
    assert_parity(s.run_component(4, h, h2), orc.fusion_proj(h, h2)[0], 1e-4, 0.99999, "fusion_proj")
    assert_parity(s.run_component(5, h, h2), orc.dit_proj(h, h2), 1e-4, 0.99999, "dit_proj")
    assert_parity(s.run_component(6, h), orc.stop_head(h), 1e-5, 0.9999, "stop_head")
    assert_parity(s.run_component(7, lat), orc.feat_encoder(lat), 1e-4, 0.99999, "feat_encoder")
    ids = synthetic.token_ids(cfg, 5, seed=4)
    assert np.array_equal(s.text_embed(ids), orc.text_embed(ids))
    s.close()


# ---------------------------------------------------------------------- DiT ---
@pytest.mark.parametrize("name", ["tiny", "bench"])
@pytest.mark.parametrize("generic", [False, True])
@pytest.mark.parametrize("plan", ["throughput", "latency"])
def test_dit_estimator(rt, models, name, generic, plan):
    """One estimator evaluation against the oracle. The latency plan gives the bench
    model's down projection a 16-CTA K split, so its residual epilogue leaves 128
    sums-of-squares parts for the next layer's q/k/v row scale."""
    cfg, blobs, dev, orc = models(name)
    s = rt.Stream(dev, kv_capacity=16)
    if plan == "latency":
        s.set_plan(rt.PLAN_LATENCY)
    rng = np.random.default_rng(21)
    x = rng.standard_normal((2, cfg.latent), dtype=np.float32)
    cond = rng.standard_normal((2, cfg.latent), dtype=np.float32)
    mu = np.zeros((2, 2 * cfg.dit_hidden), np.float32)
    mu[0] = rng.standard_normal(2 * cfg.dit_hidden)
    dt = np.zeros(2, np.float32)
    if generic:  # rows that differ in every input, as the graph contract allows
        mu[1] = rng.standard_normal(2 * cfg.dit_hidden)
        dt = np.array([0.1, 0.3], np.float32)
    else:  # what cfm_sample binds: identical x and cond rows, zero uncond mu
        x[1] = x[0]
        cond[1] = cond[0]
    t_in = np.array([4.0, 10.0], np.float32)
    want = orc.dit_estimator(x, mu, t_in, cond, dt)
    got = s.dit_estimator(x, mu, t_in, cond, dt)
    assert_parity(got, want, 2e-3 * max(1.0, float(np.abs(want).max())), 0.99999, f"{name} dit")
    s.close()


@pytest.mark.parametrize("name", ["tiny", "bench"])
def test_cfm_sample(rt, models, name):
    cfg, blobs, dev, orc = models(name)
    s = rt.Stream(dev, kv_capacity=16)
    rng = np.random.default_rng(5)
    mu = rng.standard_normal(2 * cfg.dit_hidden, dtype=np.float32)
    cond = rng.standard_normal(cfg.latent, dtype=np.float32)
    noise = oracle.noise_table(0, 1, cfg.latent)[0]
    for T in (1, 4, 10):
        want = orc.cfm_sample(mu, cond, noise, T, 2.0)
        got = s.cfm_sample(mu, cond, noise, T, 2.0)
        assert_parity(got, want, 2e-2, 0.999, f"{name} cfm T={T}")
        if T == 1:  # zero-init skip: no estimator call, the sample is the noise
            assert np.array_equal(got, noise)
    s.close()
