"""Build libvoxcpm2_cuda.so in-tree with nvcc for sm_100a (B200).

python -m voxcpm2_b200.build [--force] [-v]
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libvoxcpm2_cuda.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# host code: no FMA contraction, so the noise draws (std::normal_distribution) and the
# CFM schedule round exactly as the reference's C++ does.
FLAGS = ["-O3", "-lineinfo", "-std=c++20", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC,-fvisibility=hidden,-ffp-contract=off",
         "-ccbin", "/usr/bin/g++", f"-I{ROOT / 'include'}"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    objs, jobs = [], []
    for src in sources():
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append([NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for err in ex.map(run, jobs):
            if verbose and err:
                print(err)
    if force or jobs or _stale(LIB, objs):
        run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)])
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
