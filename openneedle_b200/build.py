"""Builds libneedle2_b200.so in-tree with nvcc for sm_100a.

The library is self-contained (static CUDA runtime, no torch), so that it can be
loaded by ctypes from any host program, including OpenNeedle's own
needle2/native.py via NEEDLE2_NATIVE_LIBRARY.
"""
from __future__ import annotations

import os
import shutil
from concurrent.futures import ThreadPoolExecutor
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libneedle2_b200.so"
INCLUDE = PKG.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fno-fast-math",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    objdir = PKG.parent / "_build" / "obj"
    objdir.mkdir(parents=True, exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    newest_header = max((p.stat().st_mtime for p in headers), default=0.0)
    jobs, objs = [], []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        objs.append(str(obj))
        # an object is reused only when it is newer than its source and every header
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            jobs.append([nvcc(), *ARCH, *FLAGS, "-dc", str(src), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for f in [pool.submit(run, cmd) for cmd in jobs]:
            f.result()
    tmp = LIB.with_suffix(".so.tmp")
    run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
