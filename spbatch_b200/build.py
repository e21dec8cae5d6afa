"""Builds libspbatch_b200.so in-tree from spbatch_b200/csrc with nvcc (sm_100a).

    python -m spbatch_b200.build          # incremental
    python -m spbatch_b200.build --force  # rebuild everything

Each .cu is compiled to an object under spbatch_b200/_build (in parallel) and
linked into spbatch_b200/libspbatch_b200.so next to this file, so the library
travels with the source tree to the GPU host.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libspbatch_b200.so")
# The same library with the test hooks of include/spb_debug.h (only api.cu
# differs); loaded by the failure-path tests, never by the product path.
DEBUG_LIB = os.path.join(PKG, "libspbatch_b200_debug.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_newer(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "**", "*.h*"), recursive=True)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool, verbose_ptxas: bool, debug: bool = False) -> str:
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ("_debug.o" if debug else ".o"))
    if force or _deps_newer(src, obj):
        cmd = [nvcc(), *ARCH, *FLAGS, *(["-DSPB_DEBUG_HOOKS"] if debug else []), "-c", src, "-o", obj]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.check_call(cmd)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), srcs))
    dbg = _compile(os.path.join(CSRC, "api.cu"), force, False, debug=True)
    dobjs = [dbg if os.path.basename(o) == "api.o" else o for o in objs]
    for lib, ob in ((LIB, objs), (DEBUG_LIB, dobjs)):
        if force or not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in ob):
            subprocess.check_call([nvcc(), *ARCH, "-shared", "-o", lib, *ob, "-lcuda", "-lcublasLt"])
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print register/smem usage (-Xptxas -v)")
    a = ap.parse_args()
    print(build(a.force, a.ptxas))
    sys.exit(0)
