"""The persistent decoder step (VXC_DECODE_STEP=persistent: every layer of one
KV-cache step in one cooperative launch) against the oracle, through the C ABI.

Same bar as the chained form: decoder outputs within max-abs 2e-2 / cosine
0.999, cache rows within 1e-4 relative; plus bit-identical reruns and the
patch loop on top of it.
"""
from __future__ import annotations

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


def persistent_stream(rt, dev, cap, monkeypatch):
    monkeypatch.setenv("VXC_DECODE_STEP", "persistent")
    s = rt.Stream(dev, kv_capacity=cap)
    monkeypatch.delenv("VXC_DECODE_STEP")
    return s


@pytest.mark.parametrize("name", ["tiny", "small", "bench"])
@pytest.mark.parametrize("which", [0, 1])
def test_persistent_step_matches_oracle(rt, models, monkeypatch, name, which):
    """Prefill 9 rows (the row path), then 6 one-token steps in the persistent form;
    the KV rows it appends are read back against the oracle's cache."""
    cfg, blobs, dev, orc = models(name)
    s = persistent_stream(rt, dev, 64, monkeypatch)
    rng = np.random.default_rng(17 + which)
    pre = rng.standard_normal((9, cfg.hidden), dtype=np.float32)
    orc.reset()
    assert_parity(s.decoder_step(which, pre), orc.decoder_forward(which, pre), 2e-2, 0.999, f"{name} prefill")
    for step in range(6):
        x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
        assert_parity(s.decoder_step(which, x), orc.decoder_forward(which, x), 2e-2, 0.999, f"{name} step {step}")
        assert s.token_count(which) == 10 + step
    layers = cfg.base_layers if which == 0 else cfg.res_layers
    for layer in (0, layers - 1):
        gk, gv = s.read_cache(which, layer)
        wk, wv = orc.read_cache(which, layer)
        assert gk.shape == wk.shape == (cfg.kv_heads, 15, cfg.head_dim)
        assert np.abs(gk - wk).max() <= 1e-4 * max(1.0, np.abs(wk).max())
        assert np.abs(gv - wv).max() <= 1e-4 * max(1.0, np.abs(wv).max())
    s.close()


def test_persistent_step_base_config_length(rt, models, monkeypatch):
    """The base decoder's configuration in the persistent form: 256 prefilled token
    ids, then 200 steps (KV 256 -> 456), every step against the oracle; the last
    splits of the attention run over more than 128 cached keys at the end."""
    cfg, blobs, dev, orc = models("bench")
    s = persistent_stream(rt, dev, 512, monkeypatch)
    ids = synthetic.token_ids(cfg, 456, seed=202)
    emb = orc.text_embed(ids)
    orc.reset()
    assert_parity(s.decoder_step(0, emb[:256]), orc.decoder_forward(0, emb[:256]), 2e-2, 0.999, "prefill")
    worst = (0.0, 1.0)
    for step in range(200):
        x = emb[256 + step: 257 + step]
        err, cos = assert_parity(s.decoder_step(0, x), orc.decoder_forward(0, x), 2e-2, 0.999, f"step {step}")
        worst = (max(worst[0], err), min(worst[1], cos))
    print(f"persistent base decoder, 200 steps: worst max-abs {worst[0]:.3e}, cosine {worst[1]:.6f}")
    gk, _ = s.read_cache(0, cfg.base_layers - 1)
    wk, _ = orc.read_cache(0, cfg.base_layers - 1)
    assert gk.shape == wk.shape and np.abs(gk - wk).max() <= 1e-4 * max(1.0, np.abs(wk).max())
    s.close()


def test_persistent_step_long_cache_sub_chunks(rt, models, monkeypatch):
    """A cache longer than 4 x 128 rows: each attention split walks its keys in
    several shared-memory sub-chunks (online softmax across them)."""
    cfg, blobs, dev, orc = models("tiny")
    s = persistent_stream(rt, dev, 1100, monkeypatch)
    rng = np.random.default_rng(5)
    pre = rng.standard_normal((1000, cfg.hidden), dtype=np.float32)
    orc.reset()
    s.decoder_step(0, pre)
    orc.decoder_forward(0, pre)
    for step in range(3):
        x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
        assert_parity(s.decoder_step(0, x), orc.decoder_forward(0, x), 2e-2, 0.999, f"step {step} over 1000+ keys")
    s.close()


def test_persistent_step_is_deterministic_and_profiles(rt, models, monkeypatch):
    """Two streams fed the same rows give bit-identical outputs; the step profile
    (a graph of cooperative launches on a private control block) leaves the
    stream's state alone."""
    cfg, blobs, dev, orc = models("small")
    a = persistent_stream(rt, dev, 64, monkeypatch)
    b = persistent_stream(rt, dev, 64, monkeypatch)
    rng = np.random.default_rng(9)
    rows = rng.standard_normal((12, cfg.hidden), dtype=np.float32)
    for s in (a, b):
        s.decoder_step(0, rows[:4])
    for i in range(4, 12):
        assert np.array_equal(a.decoder_step(0, rows[i:i + 1]), b.decoder_step(0, rows[i:i + 1]))
    before = a.token_count(0)
    ms, nb = a.profile_kernel("base_step", 5)
    assert ms > 0 and nb > 2 * cfg.base_layers * 3 * cfg.ffn * cfg.hidden
    assert a.token_count(0) == before
    x = rows[3:4]
    assert np.array_equal(a.decoder_step(0, x), b.decoder_step(0, x))
    a.close()
    b.close()


def test_persistent_step_patch_loop(rt, models, monkeypatch):
    """The whole patch loop (both decoder steps per patch in the persistent form,
    captured in the patch graph) against the oracle on TINY."""
    cfg, blobs, dev, orc = models("tiny")
    s = persistent_stream(rt, dev, 128, monkeypatch)
    ids = synthetic.token_ids(cfg, 12, seed=9)
    want = orc.generate(ids, min_patches=6, timesteps=10, cfg_value=2.0, max_patches_override=30, seed=0)
    got = s.generate(ids, min_patches=6, timesteps=10, cfg_value=2.0, max_patches_override=30, seed=0)
    assert got["patches"] == want["patches"]
    for key in ("latents", "lm_hidden", "res_hidden"):
        err = max(close_stats(got[key][i], want[key][i])[0] for i in range(got["patches"]))
        assert err <= 2e-2, (key, err)
    s.close()
