"""Builds libdvs_b200.so (the C-ABI library) in-tree for sm_100a.

    python -m dvstor_b200.build          # or: from dvstor_b200.build import build; build()

nvcc compiles every .cu/.cpp under csrc/ with -gencode arch=compute_100a,code=sm_100a
and links one shared library into dvstor_b200/lib/.  The CUDA runtime is linked
statically, so the library has no dependency on the caller's CUDA install
beyond the driver.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libdvs_b200.so")
BUILD_DIR = os.path.join(ROOT, "_build", "dvs_b200")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(target, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs, hdrs = _sources(), _headers()
    common = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"),
              "-I", CSRC]
    objs = []
    for s in srcs:
        obj = os.path.join(BUILD_DIR, os.path.basename(s) + ".o")
        objs.append(obj)
        if force or _stale(obj, [s] + hdrs):
            cmd = [nvcc()] + ARCH + common + ["-c", s, "-o", obj]
            if s.endswith(".cu"):
                cmd += ["-Xptxas", "-v"] if verbose else []
            else:
                cmd = [nvcc()] + ARCH + common + ["-x", "c++", "-c", s, "-o", obj]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-lpthread"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
