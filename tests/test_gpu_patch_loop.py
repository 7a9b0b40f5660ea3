"""GPU parity of the whole patch loop against the CPU oracle, and its failure handling.

The bar (from the task's parity contract): identical stop decisions and patch
counts; per-patch latents and hidden states within max-abs 2e-2 and cosine >= 0.999.
Failure handling is exercised from the host only: bad arguments, capacity,
cancellation (callback and another thread), non-finite estimator output.
"""
from __future__ import annotations

import threading

import numpy as np
import pytest

import oracle
from conftest import close_stats
from voxcpm2_b200 import synthetic
from voxcpm2_b200.config import BENCH, DIT_ESTIMATOR, TINY

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from voxcpm2_b200 import runtime
    return runtime


@pytest.fixture(scope="module")
def tiny(rt):
    blobs = synthetic.model_blobs(TINY, 0)
    dev = rt.Device(TINY, 0, blobs)
    yield TINY, blobs, dev, oracle.Oracle(TINY, blobs)
    dev.close()


@pytest.fixture(scope="module")
def bench(rt):
    blobs = synthetic.model_blobs(BENCH, 0)
    dev = rt.Device(BENCH, 0, blobs)
    yield BENCH, blobs, dev, oracle.Oracle(BENCH, blobs)
    dev.close()


def compare_runs(got, want, what, min_patches):
    """Identical patch count and stop decisions; every per-patch latent and hidden
    state within max-abs 2e-2 and cosine >= 0.999. Reports the worst patch."""
    n = min(got["patches"], want["patches"])
    worst = {}
    for key in ("latents", "lm_hidden", "res_hidden"):
        stats = [close_stats(got[key][i], want[key][i]) for i in range(n)]
        worst[key] = (max(s[0] for s in stats), min(s[1] for s in stats))
    decisions_g = [bool(l[1] > l[0]) for l in got["stop_logits"][:n]]
    decisions_w = [bool(l[1] > l[0]) for l in want["stop_logits"][:n]]
    margin = float(np.min(np.abs(want["stop_logits"][:n, 1] - want["stop_logits"][:n, 0])))
    summary = f"{what}: patches {got['patches']}/{want['patches']}, worst {worst}, min stop margin {margin:.2e}"
    print(summary)
    assert got["patches"] == want["patches"], summary
    assert decisions_g[min_patches + 1:] == decisions_w[min_patches + 1:], summary
    for key, (err, cos) in worst.items():
        assert err <= 2e-2 and cos >= 0.999, summary


def test_generate_tiny_full_loop(rt, tiny):
    cfg, blobs, dev, orc = tiny
    s = rt.Stream(dev, kv_capacity=128)
    ids = synthetic.token_ids(cfg, 12, seed=9)
    want = orc.generate(ids, min_patches=6, timesteps=10, cfg_value=2.0, max_patches_override=60, seed=0)
    got = s.generate(ids, min_patches=6, timesteps=10, cfg_value=2.0, max_patches_override=60, seed=0)
    compare_runs(got, want, "tiny", 6)
    assert got["patches"] >= 8
    s.close()


def test_generate_with_rope_factors(rt):
    """LongRoPE short factors (model.json setting.rope) through the whole captured
    patch loop: prefill rows and every decode step rotate as the oracle's
    make_rope_cache restatement does."""
    cfg = TINY
    blobs = synthetic.model_blobs(cfg, 0)
    dev = rt.Device(cfg, 0, blobs)
    orc = oracle.Oracle(cfg, blobs)
    short = np.random.default_rng(9).uniform(0.5, 3.0, cfg.head_dim // 2).astype(np.float32)
    dev.set_rope_factors(short)
    orc.set_rope_factors(short)
    s = rt.Stream(dev, kv_capacity=128)
    ids = synthetic.token_ids(cfg, 12, seed=2)
    want = orc.generate(ids, min_patches=6, timesteps=10, cfg_value=2.0, max_patches_override=24, seed=1)
    got = s.generate(ids, min_patches=6, timesteps=10, cfg_value=2.0, max_patches_override=24, seed=1)
    compare_runs(got, want, "tiny with rope factors", 6)
    s.close()
    dev.close()


def test_generate_bench_first_patches(rt, bench):
    """The benchmark model: 64 text tokens, the first 10 patches of the loop."""
    cfg, blobs, dev, orc = bench
    s = rt.Stream(dev, kv_capacity=512)
    ids = synthetic.token_ids(cfg, 64, seed=1)
    want = orc.generate(ids, min_patches=100, timesteps=10, cfg_value=2.0, max_patches_override=10, seed=0)
    got = s.generate(ids, min_patches=100, timesteps=10, cfg_value=2.0, max_patches_override=10, seed=0)
    compare_runs(got, want, "bench", 100)
    st = s.state()
    assert st.prefix_len == 65 and st.patches == 10
    assert st.kv_len[0] == st.kv_len[1] == 65 + 10
    s.close()


def test_latency_plan_matches_oracle(rt, bench):
    """vxc_stream_set_plan(VXC_PLAN_LATENCY) mid-utterance: the next patches run on ~296
    CTAs per estimator linear with a 3-stage ring and still meet the bar against the
    oracle; switching back is allowed; the plan cannot change with a patch in flight."""
    cfg, blobs, dev, orc = bench
    ids = synthetic.token_ids(cfg, 64, seed=1)
    want = orc.generate(ids, min_patches=100, timesteps=10, cfg_value=2.0, max_patches_override=6, seed=0)
    s = rt.Stream(dev, kv_capacity=512)
    s.prefill(ids)
    noise = oracle.noise_table(0, 6, cfg.latent)
    lat = []
    for step in range(6):
        if step == 2:
            s.set_plan(rt.PLAN_LATENCY)
        if step == 4:
            s.set_plan(rt.PLAN_THROUGHPUT)
        x, stop = s.patch_step(noise[step], min_patches=100, step=step, cfg_value=2.0, timesteps=10)
        lat.append(x)
        assert not stop
    for i in range(6):
        err = float(np.abs(lat[i] - want["latents"][i]).max())
        assert err <= 2e-2, f"patch {i}: max-abs {err:.3e}"
    with pytest.raises(rt.VxcError) as e:
        s.set_plan(7)
    assert e.value.status == 1
    s.patch_submit(noise[0], 100, 2.0, 10)
    with pytest.raises(rt.VxcError) as e:
        s.set_plan(rt.PLAN_LATENCY)  # a submitted patch is not collected yet
    assert e.value.status == 2
    s.patch_collect()
    s.close()


def test_patch_step_matches_generate(rt, tiny):
    cfg, blobs, dev, orc = tiny
    ids = synthetic.token_ids(cfg, 8, seed=2)
    a = rt.Stream(dev, kv_capacity=64)
    ref = a.generate(ids, min_patches=3, timesteps=6, cfg_value=2.0, max_patches_override=20, seed=5)
    b = rt.Stream(dev, kv_capacity=64)
    b.prefill(ids)
    noise = oracle.noise_table(5, 20, cfg.latent)
    lat = []
    for step in range(ref["patches"]):
        x, stop = b.patch_step(noise[step], min_patches=3, step=step, cfg_value=2.0, timesteps=6)
        lat.append(x)
        if stop:
            break
    assert len(lat) == ref["patches"]
    assert np.array_equal(np.stack(lat), ref["latents"])
    # device-resident driving replays the same graph from an uploaded noise table
    c = rt.Stream(dev, kv_capacity=64)
    c.prefill(ids)
    c.upload_noise(noise)
    for _ in range(ref["patches"]):
        c.patch_step_async(3, 2.0, 6)
    c.synchronize()
    st = c.state()
    assert st.patches == ref["patches"]
    assert np.array_equal(c.latents(0, ref["patches"]), ref["latents"])
    for s in (a, b, c):
        s.close()


def test_streams_run_concurrently(rt, tiny):
    cfg, blobs, dev, orc = tiny
    ids = synthetic.token_ids(cfg, 8, seed=3)
    ref = rt.Stream(dev, kv_capacity=64).generate(ids, min_patches=2, timesteps=5, max_patches_override=12, seed=1)
    streams = [rt.Stream(dev, kv_capacity=64) for _ in range(4)]
    results = [None] * 4

    def run(i):
        results[i] = streams[i].generate(ids, min_patches=2, timesteps=5, max_patches_override=12, seed=1)

    threads = [threading.Thread(target=run, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for r in results:
        assert r["patches"] == ref["patches"]
        assert np.array_equal(r["latents"], ref["latents"])
    for s in streams:
        s.close()


# ------------------------------------------------------------- failures ---
def test_step_must_follow_patch_count(rt, tiny):
    cfg, blobs, dev, orc = tiny
    s = rt.Stream(dev, kv_capacity=32)
    with pytest.raises(rt.VxcError) as e:
        s.patch_step(np.zeros(cfg.latent, np.float32), 2, 0)
    assert e.value.status == 2  # INVALID_STATE: no prefill yet
    s.prefill(synthetic.token_ids(cfg, 4, seed=0))
    with pytest.raises(rt.VxcError) as e:
        s.patch_step(np.zeros(cfg.latent, np.float32), 2, 3)
    assert e.value.status == 2
    s.patch_step(np.zeros(cfg.latent, np.float32), 2, 0)
    s.close()


def test_capacity_overflow_rejected_before_launch(rt, tiny):
    cfg, blobs, dev, orc = tiny
    s = rt.Stream(dev, kv_capacity=20)
    ids = synthetic.token_ids(cfg, 8, seed=0)
    with pytest.raises(rt.VxcError) as e:  # 9 prefix rows + 58 patches > 20
        s.generate(ids, min_patches=2, timesteps=4)
    assert e.value.status == 1
    r = s.generate(ids, min_patches=2, timesteps=4, max_patches_override=10)  # the stream is still usable
    assert 1 <= r["patches"] <= 10
    s.close()


def test_cancel_from_progress_callback(rt, tiny):
    cfg, blobs, dev, orc = tiny
    s = rt.Stream(dev, kv_capacity=128)
    seen = []

    def progress(done, total):
        seen.append(done)
        return done < 3

    with pytest.raises(rt.VxcError) as e:
        s.generate(synthetic.token_ids(cfg, 8, seed=0), min_patches=50, timesteps=4, progress=progress)
    assert e.value.status == 3
    assert seen[-1] == 3 and s.state().patches == 3
    s.close()


def test_cancel_from_another_thread(rt, tiny):
    cfg, blobs, dev, orc = tiny
    s = rt.Stream(dev, kv_capacity=128)
    started = threading.Event()

    def progress(done, total):
        if done == 2:
            started.set()
            threading.Event().wait(0.05)
        return True

    err = []

    def run():
        try:
            s.generate(synthetic.token_ids(cfg, 8, seed=0), min_patches=50, timesteps=4, progress=progress)
        except rt.VxcError as e:
            err.append(e.status)

    t = threading.Thread(target=run)
    t.start()
    started.wait(30)
    s.cancel()
    t.join(60)
    assert err == [3]
    s.close()


def test_non_finite_estimator_output_raises(rt):
    """A NaN planted in the DiT out_proj bias (host-side input) must raise, as synthesizer.cpp:150 does."""
    from voxcpm2_b200.config import DIT_ESTIMATOR, component_offsets
    blobs = synthetic.model_blobs(TINY, 0)
    off, _ = component_offsets(TINY, DIT_ESTIMATOR)["out_proj.bias"]
    blobs[DIT_ESTIMATOR] = blobs[DIT_ESTIMATOR].copy()
    blobs[DIT_ESTIMATOR][off] = np.float16(np.nan)
    dev = rt.Device(TINY, 0, blobs)
    s = rt.Stream(dev, kv_capacity=32)
    rng = np.random.default_rng(0)
    with pytest.raises(rt.VxcError) as e:
        s.cfm_sample(rng.standard_normal(2 * TINY.dit_hidden), np.zeros(TINY.latent), rng.standard_normal(TINY.latent), 4)
    assert e.value.status == 5 and "non-finite" in str(e.value)
    s.prefill(synthetic.token_ids(TINY, 4, seed=0))
    with pytest.raises(rt.VxcError) as e:
        s.patch_step(np.zeros(TINY.latent, np.float32), 2, 0)
    assert "non-finite" in str(e.value)
    s.close()
    dev.close()


def test_dit_layer_forms_agree(rt, bench, monkeypatch):
    """Both forms of the DiT decoder layers match the oracle: RMSNorm folded into
    the neighbouring tensor-core linears after layer 0 (the default, 5 launches per
    layer) and separate RMSNorm kernels (VXC_NORM_KERNELS=1, 7 launches)."""
    cfg, blobs, dev, orc = bench
    ids = synthetic.token_ids(cfg, 16, seed=4)
    want = orc.generate(ids, min_patches=100, timesteps=10, cfg_value=2.0, max_patches_override=3, seed=2)
    streams = {}
    for form, env in (("split", {}), ("split_norm_kernels", {"VXC_NORM_KERNELS": "1"})):
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        streams[form] = rt.Stream(dev, kv_capacity=64)
        for k in env:
            monkeypatch.delenv(k)
    for form, s in streams.items():
        got = s.generate(ids, min_patches=100, timesteps=10, cfg_value=2.0, max_patches_override=3, seed=2)
        compare_runs(got, want, f"{form} DiT layers", 100)
    n_layers, evals = cfg.dit_layers, 9
    k = {form: s.state().graph_kernels for form, s in streams.items()}
    assert k["split_norm_kernels"] - k["split"] == (2 * n_layers - 1) * evals
    for s in streams.values():
        s.close()


def test_time_tables_follow_weight_reload(rt, tiny):
    """The per-T time-token tables are derived from the DiT weights: a reload of
    those weights must show up in the next patch."""
    cfg, blobs, _, _ = tiny
    dev = rt.Device(cfg, 0, blobs)
    s = rt.Stream(dev, kv_capacity=64)
    ids = synthetic.token_ids(cfg, 8, seed=6)
    s.generate(ids, min_patches=2, timesteps=6, cfg_value=2.0, max_patches_override=3, seed=3)
    other = synthetic.model_blobs(cfg, 1)
    dit = DIT_ESTIMATOR
    dev.load(dit, other[dit])
    mixed = dict(blobs)
    mixed[dit] = other[dit]
    want = oracle.Oracle(cfg, mixed).generate(ids, min_patches=2, timesteps=6, cfg_value=2.0,
                                              max_patches_override=3, seed=3)
    got = s.generate(ids, min_patches=2, timesteps=6, cfg_value=2.0, max_patches_override=3, seed=3)
    compare_runs(got, want, "after DiT weight reload", 2)
    s.close()
    dev.close()


def test_decode_step_profile_keeps_stream_state(rt, tiny):
    """The whole-step and whole-evaluation profiles run on a private control block
    and write their output to scratch: the stream's KV lengths and its next patch
    are unaffected."""
    cfg, blobs, dev, orc = tiny
    ids = synthetic.token_ids(cfg, 8, seed=4)
    noise = oracle.noise_table(6, 4, cfg.latent)
    a = rt.Stream(dev, kv_capacity=64)
    a.prefill(ids)
    a.patch_step(noise[0], min_patches=10, step=0, cfg_value=2.0, timesteps=5)
    before = a.state()
    for k in ("base_step", "res_step", "dit_eval"):
        ms, nb = a.profile_kernel(k, 5)
        assert ms > 0
        if k == "dit_eval":
            assert nb > 2 * cfg.dit_layers * 3 * cfg.dit_ffn * cfg.dit_hidden  # at least the MLP weights
        else:
            layers = cfg.base_layers if k == "base_step" else cfg.res_layers
            assert nb > 2 * layers * 3 * cfg.ffn * cfg.hidden
    after = a.state()
    assert (after.kv_len[0], after.kv_len[1], after.patches) == (before.kv_len[0], before.kv_len[1], before.patches)
    x1, _ = a.patch_step(noise[1], min_patches=10, step=1, cfg_value=2.0, timesteps=5)
    b = rt.Stream(dev, kv_capacity=64)
    b.prefill(ids)
    b.patch_step(noise[0], min_patches=10, step=0, cfg_value=2.0, timesteps=5)
    y1, _ = b.patch_step(noise[1], min_patches=10, step=1, cfg_value=2.0, timesteps=5)
    assert np.array_equal(x1, y1)
    a.close()
    b.close()


def test_shared_receive_buffer_is_bit_identical(rt, bench, monkeypatch):
    """VXC_RECV_SHARED=1 only moves the split-K receive buffer into the stage area
    (same rank-order sums): the latents are bit-identical to the default's."""
    cfg, blobs, dev, orc = bench
    ids = synthetic.token_ids(cfg, 16, seed=8)
    a = rt.Stream(dev, kv_capacity=64)
    monkeypatch.setenv("VXC_RECV_SHARED", "1")
    b = rt.Stream(dev, kv_capacity=64)
    monkeypatch.delenv("VXC_RECV_SHARED")
    ra = a.generate(ids, min_patches=100, timesteps=10, cfg_value=2.0, max_patches_override=3, seed=4, trace=False)
    rb = b.generate(ids, min_patches=100, timesteps=10, cfg_value=2.0, max_patches_override=3, seed=4, trace=False)
    assert np.array_equal(ra["latents"], rb["latents"])
    a.close()
    b.close()


def _run_prefix(rt, dev, cfg, rows, flags, audio, seed, patches, timesteps):
    s = rt.Stream(dev, kv_capacity=128)
    s.prefill_rows(rows, flags, audio)
    s.upload_noise(oracle.noise_table(seed, patches, cfg.latent))
    for _ in range(patches):
        s.patch_step_async(1000, 2.0, timesteps)
    s.synchronize()
    st = s.state()
    assert st.prefix_len == len(rows) and st.patches == patches
    lat = s.latents(0, patches)
    s.close()
    return lat


@pytest.mark.parametrize("layout", ["prompt_audio_last", "reference_audio_inside"])
def test_prefill_rows_with_audio_matches_oracle(rt, tiny, layout):
    """Prefixes with audio rows (synthesizer.cpp:359-535): feat_encoder embeddings,
    FSQ'd LM rows, the residual feature input, and the first patch's condition
    (the last prompt patch, or zeros when the prefix ends in a token)."""
    cfg, blobs, dev, orc = tiny
    text = synthetic.token_ids(cfg, 7, seed=31)
    audio = np.random.default_rng(3).standard_normal((3, cfg.latent)).astype(np.float32)
    if layout == "prompt_audio_last":
        rows = np.concatenate([text, [cfg.audio_start_token, 0, 0, 0]]).astype(np.int32)
        flags = np.array([0] * (text.size + 1) + [1, 1, 1], np.int32)
        aud = audio
    else:  # reference audio between two marker tokens, then the target text
        rows = np.concatenate([[102, 0, 0, 103], text, [cfg.audio_start_token]]).astype(np.int32)
        flags = np.array([0, 1, 1, 0] + [0] * (text.size + 1), np.int32)
        aud = audio[:2]
    got = _run_prefix(rt, dev, cfg, rows, flags, aud, seed=12, patches=6, timesteps=6)
    want = orc.generate_rows(rows, flags, aud, text.size, min_patches=1000, timesteps=6, max_patches_override=6,
                             seed=12)
    assert want["patches"] == 6
    for i in range(6):
        err, cos = close_stats(got[i], want["latents"][i])
        assert err <= 2e-2 and cos >= 0.999, (layout, i, err, cos)


def test_prefill_rows_text_only_is_prefill(rt, tiny):
    """A row prefix of the text ids + audio_start and no audio rows is vxc_prefill's."""
    cfg, blobs, dev, orc = tiny
    text = synthetic.token_ids(cfg, 9, seed=32)
    rows = np.append(text, cfg.audio_start_token).astype(np.int32)
    a = _run_prefix(rt, dev, cfg, rows, None, None, seed=3, patches=3, timesteps=5)
    s = rt.Stream(dev, kv_capacity=128)
    s.prefill(text)
    s.upload_noise(oracle.noise_table(3, 3, cfg.latent))
    for _ in range(3):
        s.patch_step_async(1000, 2.0, 5)
    s.synchronize()
    assert np.array_equal(a, s.latents(0, 3))
    with pytest.raises(rt.VxcError):
        s.prefill_rows(rows, np.ones(rows.size, np.int32), None)  # audio rows without latents
    s.close()


def test_prefill_rows_bench_model(rt, bench):
    cfg, blobs, dev, orc = bench
    text = synthetic.token_ids(cfg, 24, seed=33)
    audio = np.random.default_rng(4).standard_normal((4, cfg.latent)).astype(np.float32)
    rows = np.concatenate([text, [cfg.audio_start_token, 0, 0, 0, 0]]).astype(np.int32)
    flags = np.array([0] * (text.size + 1) + [1] * 4, np.int32)
    got = _run_prefix(rt, dev, cfg, rows, flags, audio, seed=21, patches=3, timesteps=10)
    want = orc.generate_rows(rows, flags, audio, text.size, min_patches=1000, timesteps=10, max_patches_override=3,
                             seed=21)
    for i in range(3):
        err, cos = close_stats(got[i], want["latents"][i])
        assert err <= 2e-2 and cos >= 0.999, (i, err, cos)


def test_pipelined_submit_collect_matches_patch_step(rt, tiny):
    """vxc_patch_submit / vxc_patch_collect with one patch queued ahead give the
    synchronous vxc_patch_step's latents and stop flags, bit for bit."""
    cfg, blobs, dev, orc = tiny
    ids = synthetic.token_ids(cfg, 8, seed=14)
    noise = oracle.noise_table(17, 10, cfg.latent)
    a = rt.Stream(dev, kv_capacity=64)
    a.prefill(ids)
    want = [a.patch_step(noise[i], min_patches=2, step=i, cfg_value=2.0, timesteps=5) for i in range(10)]
    b = rt.Stream(dev, kv_capacity=64)
    b.prefill(ids)
    with pytest.raises(rt.VxcError) as e:
        b.patch_collect()  # nothing queued
    assert e.value.status == 2
    got = []
    b.patch_submit(noise[0], 2, 2.0, 5)
    for i in range(1, 10):
        b.patch_submit(noise[i], 2, 2.0, 5)
        got.append(b.patch_collect())
    got.append(b.patch_collect())
    for (gl, gs), (wl, ws) in zip(got, want):
        assert np.array_equal(gl, wl) and gs == ws
    st = b.state()
    assert st.patches == 10 and st.kv_len[0] == a.state().kv_len[0]
    for i in range(4):
        b.patch_submit(noise[i], 2, 2.0, 5)
    with pytest.raises(rt.VxcError):
        b.patch_submit(noise[4], 2, 2.0, 5)  # four already in flight
    b.prefill(ids)  # drops the queued patches
    with pytest.raises(rt.VxcError):
        b.patch_collect()
    a.close()
    b.close()
