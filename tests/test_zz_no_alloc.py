"""The allocation-free SDPA entry point against the allocating one (collected last).

vxc_sdpa_decode_noalloc serves callers that must not let a library allocate
device memory (plugin hosts that forbid allocation in their enqueue call,
real-time threads that cannot absorb cudaMalloc's device synchronisation). Its
split-K scratch is a fixed device array inside the library, so two calls in a
row reuse the same memory; both must match vxc_sdpa to the SDPA tolerance of
the other tests (1e-5).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run_pair(rt, torch, rng, heads, groups, past, cur, with_mask, scale):
    d = 64
    dev = torch.device("cuda", 0)

    def t(*shape):
        return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(dev)

    q, k, v = t(heads, 1, d), t(groups, cur, d), t(groups, cur, d)
    pk = t(groups, past, d) if past else None
    pv = t(groups, past, d) if past else None
    mask = torch.zeros(1, past + cur, device=dev) if with_mask else None
    ptr = lambda x: 0 if x is None else x.data_ptr()  # noqa: E731
    outs = {}
    for name in ("alloc", "noalloc"):
        out = torch.empty(heads, 1, d, device=dev)
        ok = torch.empty(groups, past + cur, d, device=dev)
        ov = torch.empty(groups, past + cur, d, device=dev)
        if name == "alloc":
            rt.sdpa_device(ptr(q), heads, 1, d, ptr(k), ptr(v), groups, cur, d, ptr(mask), 1 if with_mask else 0,
                           ptr(pk), ptr(pv), past, scale, ptr(out), ptr(ok), ptr(ov))
        else:
            rt.sdpa_decode_noalloc(ptr(q), heads, d, ptr(k), ptr(v), groups, cur, ptr(mask), ptr(pk), ptr(pv),
                                   past, scale, ptr(out), ptr(ok), ptr(ov))
        torch.cuda.synchronize()
        outs[name] = (out.cpu().numpy(), ok.cpu().numpy(), ov.cpu().numpy())
    return outs


def test_no_alloc_sdpa_matches_allocating_sdpa_twice():
    torch = pytest.importorskip("torch")
    from voxcpm2_b200 import runtime as rt
    rng = np.random.default_rng(2024)
    # two calls in a row with different shapes: the second reuses the array the first left behind
    for heads, groups, past, cur, with_mask, scale in ((16, 2, 512, 1, True, 0.125), (32, 4, 95, 1, False, 0.0)):
        outs = _run_pair(rt, torch, rng, heads, groups, past, cur, with_mask, scale)
        a, b = outs["alloc"], outs["noalloc"]
        assert np.abs(a[0] - b[0]).max() <= 1e-5
        assert np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    pytest.importorskip("torch")
    from voxcpm2_b200 import runtime as rt
    with pytest.raises(rt.VxcError) as e:  # 128 query heads > the fixed scratch's 64
        rt.sdpa_decode_noalloc(1, 128, 64, 1, 1, 8, 1, 0, 0, 0, 0, 0.0, 1)
    assert e.value.status == 1 and "64 query heads" in str(e.value)
