"""Build libmgcuda.so in-tree (nvcc, sm_100a) -- ``python -m edge_maskgit_b200.build``.

Objects go to edge_maskgit_b200/_build/; the shared library to edge_maskgit_b200/libmgcuda.so.
Sources are recompiled only when they (or a header) are newer than their object.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libmgcuda.so"
ROOT = PKG.parent

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC",
                  "-I", str(ROOT / "include"), "--expt-relaxed-constexpr"] + \
    os.environ.get("MGC_EXTRA_NVFLAGS", "").split()


def _headers() -> list[Path]:
    return list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "mgc.h"]


def _stale(src: Path, obj: Path, hdr_mtime: float) -> bool:
    return not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_mtime)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = max(p.stat().st_mtime for p in _headers())
    jobs = []
    objs = []
    for src in sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp")):
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if _stale(src, obj, hdr):
            jobs.append([NVCC, *NVFLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(_run, jobs))
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp),
              "-cudart", "static"])
        os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


def build_oracle() -> None:
    """Compile the test-only CPU oracle (and the reference CPU path where its tree exists)."""
    _run(["make", "-s", "-C", str(ROOT / "oracle")])


if __name__ == "__main__":
    build(verbose=True)
    if "--oracle" in sys.argv:
        build_oracle()
