"""The C ABI header compiles as C11 and links against the library (no GPU needed)."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib_path():
    from voxcpm2_b200 import build
    return build.build()


def test_header_compiles_as_c11_and_links(lib_path, tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = tmp_path / "c_api_header"
    cmd = [cc, "-std=c11", "-pedantic", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
           str(ROOT / "tests" / "c" / "c_api_header.c"), "-o", str(exe), f"-L{lib_path.parent}", "-lvoxcpm2_cuda",
           f"-Wl,-rpath,{lib_path.parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert r.stdout.startswith("ok ")
