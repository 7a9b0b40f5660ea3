"""The allocation-free SDPA entry point against the oracle and the allocating one (collected last).

vxc_sdpa_decode_noalloc serves callers that must not let a library allocate
device memory (plugin hosts that forbid allocation in their enqueue call,
real-time threads that cannot absorb cudaMalloc's device synchronisation). Its
split-K scratch is a fixed device array inside the library, so calls in a row
reuse the same memory. Every call is held to the oracle (the reference layer's
CPU forward restated) at the SDPA tolerance of the other tests (1e-5), and to
vxc_sdpa on the same inputs.

The cases reach the limits the entry point documents: 64 query heads (the top
of the fixed array), 16 heads per KV group, 2048 keys (32 splits of 64 keys
each, more than the 32 keys a split takes below 1024), one head per group, and
non-zero additive masks.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

D = 64


def _inputs(rng, heads, groups, past, cur, masked):
    q = rng.standard_normal((heads, 1, D), dtype=np.float32)
    k = rng.standard_normal((groups, cur, D), dtype=np.float32)
    v = rng.standard_normal((groups, cur, D), dtype=np.float32)
    pk = rng.standard_normal((groups, past, D), dtype=np.float32) if past else None
    pv = rng.standard_normal((groups, past, D), dtype=np.float32) if past else None
    mask = (rng.standard_normal((1, past + cur)) * 2.0).astype(np.float32) if masked else None
    return q, k, v, pk, pv, mask


def _run(rt, torch, name, host, heads, groups, past, cur, scale):
    """One call of vxc_sdpa ('alloc') or vxc_sdpa_decode_noalloc ('noalloc') on device
    copies of the host inputs: (out, out_k, out_v) on the host."""
    dev = torch.device("cuda", 0)
    q, k, v, pk, pv, mask = (None if a is None else torch.from_numpy(a).to(dev) for a in host)
    ptr = lambda x: 0 if x is None else x.data_ptr()  # noqa: E731
    out = torch.empty(heads, 1, D, device=dev)
    ok = torch.empty(groups, past + cur, D, device=dev)
    ov = torch.empty(groups, past + cur, D, device=dev)
    if name == "alloc":
        rt.sdpa_device(ptr(q), heads, 1, D, ptr(k), ptr(v), groups, cur, D, ptr(mask), 1 if mask is not None else 0,
                       ptr(pk), ptr(pv), past, scale, ptr(out), ptr(ok), ptr(ov))
    else:
        rt.sdpa_decode_noalloc(ptr(q), heads, D, ptr(k), ptr(v), groups, cur, ptr(mask), ptr(pk), ptr(pv),
                               past, scale, ptr(out), ptr(ok), ptr(ov))
    torch.cuda.synchronize()
    return out.cpu().numpy(), ok.cpu().numpy(), ov.cpu().numpy()


# (heads, groups, past, cur, masked, scale); calls run in this order, each reusing the
# array the one before left behind
CASES = (
    (64, 4, 512, 1, True, 0.125),    # 513 keys, 16 heads per group, the fixed array's top head
    (64, 4, 2047, 1, True, 0.125),   # 2048 keys: 32 splits of 64 keys
    (4, 4, 2047, 1, False, 0.0),     # one head per group, default scale
    (32, 4, 95, 1, False, 0.0),      # a short row after the long ones
    (16, 2, 1200, 1, True, 0.125),   # GQA 8:1 over 1201 keys
)


def test_no_alloc_sdpa_matches_oracle_on_calls_in_a_row():
    torch = pytest.importorskip("torch")
    from voxcpm2_b200 import runtime as rt
    rng = np.random.default_rng(2024)
    for heads, groups, past, cur, masked, scale in CASES:
        host = _inputs(rng, heads, groups, past, cur, masked)
        q, k, v, pk, pv, mask = host
        want, wk, wv = oracle.sdpa(q, k, v, mask, pk, pv, scale, want_cache=True)
        what = f"heads {heads}, groups {groups}, keys {past + cur}, mask {masked}"
        for _ in range(2):  # two calls in a row on the same inputs
            got, gk, gv = _run(rt, torch, "noalloc", host, heads, groups, past, cur, scale)
            assert np.abs(got - want).max() <= 1e-5, what
            assert np.array_equal(gk, wk) and np.array_equal(gv, wv), what
        ref, _, _ = _run(rt, torch, "alloc", host, heads, groups, past, cur, scale)
        assert np.abs(got - ref).max() <= 1e-5, what


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    pytest.importorskip("torch")
    from voxcpm2_b200 import runtime as rt
    with pytest.raises(rt.VxcError) as e:  # 128 query heads > the fixed scratch's 64
        rt.sdpa_decode_noalloc(1, 128, 64, 1, 1, 8, 1, 0, 0, 0, 0, 0.0, 1)
    assert e.value.status == 1 and "64 query heads" in str(e.value)
