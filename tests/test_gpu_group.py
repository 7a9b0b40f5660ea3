"""GPU parity of stream groups: several streams stepped as one CUDA graph with
their estimator evaluations batched into one pass over the DiT weights.

Each member has its own prompt and noise table; its latents must match the
oracle's generate() for that prompt and seed at the patch-loop bar (per patch
max-abs 2e-2, cosine >= 0.999), and its KV lengths and patch count must advance
as a lone stream's do. Stop decisions are kept out of play (min_patches above
the patches run) so every member runs every patch.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import close_stats, fsq_codes_from_hidden, fsq_forced_disagreements
from voxcpm2_b200 import synthetic
from voxcpm2_b200.config import BENCH, TINY

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from voxcpm2_b200 import runtime
    return runtime


def run_group(rt, cfg, dev, prompts, seeds, patches, timesteps=10, cfg_value=2.0):
    g = rt.Group(dev, len(prompts), kv_capacity=256)
    for st, ids, seed in zip(g.streams, prompts, seeds):
        st.prefill(ids)
        st.upload_noise(oracle.noise_table(seed, patches, cfg.latent))
    for _ in range(patches):
        g.patch_step_async(10 * patches, cfg_value, timesteps)
    g.synchronize()
    out = []
    for st, ids in zip(g.streams, prompts):
        s = st.state()
        assert s.patches == patches
        assert s.kv_len[0] == s.kv_len[1] == len(ids) + 1 + patches
        out.append(st.latents(0, patches))
    kernels = g.graph_kernels()
    g.close()
    return out, kernels


def check_members(orc, prompts, seeds, got, patches, timesteps=10, cfg_value=2.0):
    for m, (ids, seed) in enumerate(zip(prompts, seeds)):
        want = orc.generate(ids, min_patches=10 * patches, timesteps=timesteps, cfg_value=cfg_value,
                            max_patches_override=patches, seed=seed)
        assert want["patches"] == patches
        stats = [close_stats(got[m][i], want["latents"][i]) for i in range(patches)]
        err, cos = max(s[0] for s in stats), min(s[1] for s in stats)
        print(f"member {m}: worst max-abs {err:.3e}, cosine {cos:.6f}")
        assert err <= 2e-2 and cos >= 0.999, (m, err, cos)


@pytest.mark.parametrize("members,bulk", [(1, "0"), (4, "0"), (4, "1"), (6, "0"), (8, "0"), (8, "1")])
def test_group_tiny_matches_oracle(rt, members, bulk, monkeypatch):
    """TINY groups of 1 to 8 members; the decoder GEMVs in the register-streaming
    batch form (the default) and in the bulk-copy form (VXC_GROUP_BULK_GEMV=1).
    Groups of 5 to 8 members run the wide linears on a 144- or 176-row block (256
    TMEM columns, N = 144 / 176 MMAs) and the 8-slot member batches."""
    monkeypatch.setenv("VXC_GROUP_BULK_GEMV", bulk)
    blobs = synthetic.model_blobs(TINY, 0)
    dev = rt.Device(TINY, 0, blobs)
    orc = oracle.Oracle(TINY, blobs)
    prompts = [synthetic.token_ids(TINY, 6 + 3 * m, seed=20 + m) for m in range(members)]
    seeds = [100 + m for m in range(members)]
    got, kernels = run_group(rt, TINY, dev, prompts, seeds, patches=8, timesteps=6)
    check_members(orc, prompts, seeds, got, 8, timesteps=6)
    assert kernels > 0
    dev.close()


def test_group_bench_eight_members_match_oracle(rt):
    """The benchmark model, a group of 8 members (176 estimator rows per pass), 3
    patches, every member against its own oracle run.

    FSQ rounds tanh(z) * 9 to integers, and a value within float rounding of a
    half-integer can round one way on the GPU and the other on the CPU; the next
    patches then belong to different utterances. So each member is held to the
    oracle following the GPU's FSQ codes (recovered from the member's LM states),
    and every code the oracle would have rounded the other way must be a one-step
    change within 1e-3 of the rounding boundary."""
    cfg = BENCH
    blobs = synthetic.model_blobs(cfg, 0)
    dev = rt.Device(cfg, 0, blobs)
    orc = oracle.Oracle(cfg, blobs)
    patches = 3
    prompts = [synthetic.token_ids(cfg, 16 + 6 * m, seed=130 + m) for m in range(8)]
    seeds = [170 + m for m in range(8)]
    g = rt.Group(dev, 8, kv_capacity=256)
    for st, ids, seed in zip(g.streams, prompts, seeds):
        st.prefill(ids)
        st.upload_noise(oracle.noise_table(seed, patches, cfg.latent))
    lm = [[] for _ in range(8)]
    for _ in range(patches):
        for m, st in enumerate(g.streams):
            lm[m].append(st.hidden()[0])  # the LM state entering this patch
        g.patch_step_async(10 * patches, 2.0, 10)
        g.synchronize()
    for m, (st, ids, seed) in enumerate(zip(g.streams, prompts, seeds)):
        s = st.state()
        assert s.patches == patches and s.kv_len[0] == s.kv_len[1] == len(ids) + 1 + patches
        got = st.latents(0, patches)
        codes, resid = fsq_codes_from_hidden(cfg, blobs, lm[m][1:patches])
        assert resid < 1e-2, (m, resid)
        want = orc.generate(ids, min_patches=10 * patches, timesteps=10, cfg_value=2.0,
                            max_patches_override=patches, seed=seed, fsq_codes=codes)
        dis = fsq_forced_disagreements(want["fsq_pre"], codes)
        for p, j, own, c, d in dis:
            assert abs(own - c) == 1 and d < 1e-3, (m, p, j, own, c, d)
        stats = [close_stats(got[i], want["latents"][i]) for i in range(patches)]
        err, cos = max(x[0] for x in stats), min(x[1] for x in stats)
        print(f"member {m}: {len(dis)} FSQ codes rounded the other way, worst max-abs {err:.3e}, cosine {cos:.6f}")
        assert err <= 2e-2 and cos >= 0.999, (m, err, cos)
    g.close()
    dev.close()


def test_group_bench_matches_oracle(rt):
    """The benchmark model, 3 members with different prompts, 4 patches."""
    blobs = synthetic.model_blobs(BENCH, 0)
    dev = rt.Device(BENCH, 0, blobs)
    orc = oracle.Oracle(BENCH, blobs)
    prompts = [synthetic.token_ids(BENCH, n, seed=30 + n) for n in (64, 40, 17)]
    seeds = [7, 8, 9]
    got, kernels = run_group(rt, BENCH, dev, prompts, seeds, patches=4)
    check_members(orc, prompts, seeds, got, 4)
    # one estimator pass and one batched decoder step per group patch: about as
    # many launches as one lone stream's patch, not 3 times as many
    lone = rt.Stream(dev, kv_capacity=64)
    lone.prefill(prompts[2])
    lone.upload_noise(oracle.noise_table(9, 1, BENCH.latent))
    lone.patch_step_async(100, 2.0, 10)
    lone.synchronize()
    assert kernels < 2 * lone.state().graph_kernels, (kernels, lone.state().graph_kernels)
    lone.close()
    dev.close()


def test_group_orders_with_member_calls(rt):
    """Member-stream calls queued around a group step see its results without a
    group synchronize: the step waits for them and they wait for the step."""
    blobs = synthetic.model_blobs(TINY, 0)
    dev = rt.Device(TINY, 0, blobs)
    prompts = [synthetic.token_ids(TINY, 7, seed=41), synthetic.token_ids(TINY, 9, seed=42)]
    g = rt.Group(dev, 2, kv_capacity=64)
    ref, _ = run_group(rt, TINY, dev, prompts, [3, 4], patches=3, timesteps=5)
    for st, ids, seed in zip(g.streams, prompts, [3, 4]):
        st.prefill(ids)
        st.upload_noise(oracle.noise_table(seed, 3, TINY.latent))
    for _ in range(3):
        g.patch_step_async(30, 2.0, 5)
    for m, st in enumerate(g.streams):  # no g.synchronize(): read_latents is ordered on the member stream
        assert np.array_equal(st.latents(0, 3), ref[m])
    g.close()
    with pytest.raises(rt.VxcError):
        rt.Group(dev, 9, kv_capacity=64)
    dev.close()


def stop_prone_blobs():
    """TINY weights whose stop head's 'stop' row is the 'continue' row plus a
    random N(0, 0.5) vector (seed 1): the stop logit gap then has a spread of ~1,
    so decisions flip early and with clear margins (the random-init head's gap is
    ~1e-3 and never favours stopping within 24 patches)."""
    from voxcpm2_b200.config import STOP_HEAD
    blobs = dict(synthetic.model_blobs(TINY, 0))
    H = TINY.hidden
    sh = np.array(blobs[STOP_HEAD], dtype=np.float16).copy()
    off = H * H + H
    v = np.random.default_rng(1).normal(0, 0.5, H).astype(np.float32)
    sh[off + H: off + 2 * H] = (sh[off: off + H].astype(np.float32) + v).astype(np.float16)
    blobs[STOP_HEAD] = sh
    return blobs


@pytest.mark.parametrize("members", [4, 8])
def test_group_members_stop_independently(rt, members):
    """Small min_patches: members reach the stop rule at their own patches (their
    decoder steps inside the batched kernels skip once their own flag is set).
    Each member's stop patch and latents up to it match the oracle's generate()
    (with these weights the oracle stops the first four members after 5, never, 6
    and 8 patches)."""
    blobs = stop_prone_blobs()
    dev = rt.Device(TINY, 0, blobs)
    orc = oracle.Oracle(TINY, blobs)
    cap_patches = 24
    prompts = [synthetic.token_ids(TINY, 5 + 2 * m, seed=60 + m) for m in range(members)]
    seeds = [300 + m for m in range(members)]
    g = rt.Group(dev, members, kv_capacity=128)
    for st, ids, seed in zip(g.streams, prompts, seeds):
        st.prefill(ids)
        st.upload_noise(oracle.noise_table(seed, cap_patches, TINY.latent))
    first_stop = [None] * members
    for step in range(cap_patches):
        g.patch_step_async(2, 2.0, 6)
        g.synchronize()
        for m, st in enumerate(g.streams):
            if first_stop[m] is None and st.state().stopped:
                first_stop[m] = step
        if all(f is not None for f in first_stop):
            break
    for m, (st, ids, seed) in enumerate(zip(g.streams, prompts, seeds)):
        want = orc.generate(ids, min_patches=2, timesteps=6, cfg_value=2.0, max_patches_override=cap_patches,
                            seed=seed)
        got_n = cap_patches if first_stop[m] is None else first_stop[m] + 1
        assert got_n == want["patches"], (m, got_n, want["patches"])
        got = st.latents(0, got_n)
        stats = [close_stats(got[i], want["latents"][i]) for i in range(got_n)]
        err, cos = max(s[0] for s in stats), min(s[1] for s in stats)
        print(f"member {m}: stop after {got_n} patches, worst max-abs {err:.3e}, cosine {cos:.6f}")
        assert err <= 2e-2 and cos >= 0.999, (m, err, cos)
    assert sum(f is not None for f in first_stop) >= 2
    g.close()
    dev.close()


def test_group_rejects_bad_use(rt):
    """Errors come back as statuses before anything is launched: an empty group, a
    step before every member is prefilled, non-positive timesteps."""
    blobs = synthetic.model_blobs(TINY, 0)
    dev = rt.Device(TINY, 0, blobs)
    with pytest.raises(rt.VxcError):
        rt.Group(dev, 0, kv_capacity=64)
    g = rt.Group(dev, 2, kv_capacity=64)
    with pytest.raises(rt.VxcError):
        g.patch_step_async(2, 2.0, 6)  # no member prefilled
    g.streams[0].prefill(synthetic.token_ids(TINY, 6, seed=1))
    with pytest.raises(rt.VxcError):
        g.patch_step_async(2, 2.0, 6)  # member 1 not prefilled
    g.streams[1].prefill(synthetic.token_ids(TINY, 7, seed=2))
    with pytest.raises(rt.VxcError):
        g.patch_step_async(2, 2.0, 0)
    for st, seed in zip(g.streams, (5, 6)):
        st.upload_noise(oracle.noise_table(seed, 2, TINY.latent))
    g.patch_step_async(10, 2.0, 6)  # the group still works after the rejected calls
    g.synchronize()
    assert [st.state().patches for st in g.streams] == [1, 1]
    g.close()
    dev.close()


@pytest.mark.parametrize("members", [4, 8])
def test_group_receive_buffer_forms_bit_identical(rt, monkeypatch, members):
    """The wide linears' split-K partials in the stage area (the default) or in a
    dedicated buffer (VXC_GROUP_RECV_SHARED=0, where it fits beside the ring):
    same sums, identical latents."""
    blobs = synthetic.model_blobs(TINY, 0)
    dev = rt.Device(TINY, 0, blobs)
    prompts = [synthetic.token_ids(TINY, 6 + m, seed=80 + m) for m in range(members)]
    got = []
    for env in ("1", "0"):
        monkeypatch.setenv("VXC_GROUP_RECV_SHARED", env)
        lat, _ = run_group(rt, TINY, dev, prompts, [90 + m for m in range(members)], patches=4, timesteps=6)
        got.append(lat)
    for a, b in zip(*got):
        assert np.array_equal(a, b)
    dev.close()
