"""The C-ABI library: builds, loads, exports what include/voxcpm2_cuda.h declares (no GPU needed)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "voxcpm2_cuda.h"


@pytest.fixture(scope="module")
def rt():
    from voxcpm2_b200 import build
    build.build()
    from voxcpm2_b200 import runtime
    runtime.lib()
    return runtime


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"VXC_API\s+[\w\s\*]+?\b(vxc_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert "vxc_patch_step" in names and "vxc_sdpa" in names and "vxc_decoder_step" in names
    assert len(names) >= 29


def test_library_exports_every_declared_symbol(rt):
    L = rt.lib()
    for name in declared():
        assert hasattr(L, name), f"{name} declared in include/voxcpm2_cuda.h but not exported"
    assert set(declared()) == set(rt.SIGNATURES), "ctypes signatures out of sync with the header"


def test_abi_version(rt):
    assert rt.lib().vxc_abi_version() == 1


def test_component_counts_match_config(rt):
    from voxcpm2_b200.config import BENCH, COMPONENTS, SMALL, TINY, component_count
    for cfg in (TINY, SMALL, BENCH):
        d = rt.desc(cfg)
        for c in COMPONENTS:
            assert rt.lib().vxc_component_weight_count(C.byref(d), c) == component_count(cfg, c)


def test_null_arguments_are_invalid_argument(rt):
    h = C.c_void_p()
    assert rt.lib().vxc_device_create(0, None, C.byref(h)) == 1
    assert b"null" in rt.lib().vxc_last_error()
    assert rt.lib().vxc_stream_create(None, 16, C.byref(h)) == 1
    assert rt.lib().vxc_set_rope_factors(None, None, None, 32) == 1
    assert rt.lib().vxc_stream_set_plan(None, 1) == 1
    # stream groups
    assert rt.lib().vxc_group_create(None, 2, 16, C.byref(h)) == 1
    assert rt.lib().vxc_group_stream(None, 0, C.byref(h)) == 1
    assert rt.lib().vxc_group_patch_step_async(None, 1, 2.0, 10) == 1
    assert rt.lib().vxc_group_synchronize(None) == 1
    n = C.c_int32()
    assert rt.lib().vxc_group_graph_kernels(None, C.byref(n)) == 1
    rt.lib().vxc_group_destroy(None)  # a no-op


def test_bad_model_description_rejected(rt):
    from voxcpm2_b200.config import TINY
    import dataclasses
    bad = rt.desc(dataclasses.replace(TINY, head_dim=48))
    h = C.c_void_p()
    assert rt.lib().vxc_device_create(0, C.byref(bad), C.byref(h)) == 1
    assert b"head_dim" in rt.lib().vxc_last_error()


def test_no_cpu_fallback_without_device(rt):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from voxcpm2_b200.config import TINY
    with pytest.raises(rt.VxcError) as e:
        rt.Device(TINY)
    assert e.value.status == 5


def test_product_never_imports_the_oracle():
    pkg = ROOT / "voxcpm2_b200"
    for path in list(pkg.glob("*.py")) + list((pkg / "csrc").glob("*")):
        text = path.read_text(errors="ignore")
        assert "import oracle" not in text and "from oracle" not in text and "liborc" not in text, path


def test_profile_kernel_ids_match_header():
    """runtime.PROFILE_KERNELS mirrors the header's VXC_PROF_* enum."""
    import re
    from voxcpm2_b200 import runtime
    text = (ROOT / "include" / "voxcpm2_cuda.h").read_text()
    ids = {m.group(1).lower(): int(m.group(2)) for m in re.finditer(r"VXC_PROF_([A-Z_]+)\s*=\s*(\d+)", text)}
    assert ids, "no VXC_PROF_* enumerators found"
    assert runtime.PROFILE_KERNELS == ids
