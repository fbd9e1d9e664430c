"""Build recipe for the native library ``beam_engine_b200/lib/libbeam_b200.so``.

One ``nvcc`` invocation per source, sm_100a only, position-independent code,
linked into an in-tree shared library with a plain C ABI (``include/beam_b200.h``);
Python binds it with ctypes.  Run ``python -m beam_engine_b200.build_lib``.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(OUT_DIR, "libbeam_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["lib.cu"]
HOST_SOURCES = ["host/planner.cpp", "host/trie.cpp", "host/diverse.cpp"]


def _sources():
    out = []
    for s in CUDA_SOURCES + HOST_SOURCES:
        p = os.path.join(CSRC, s)
        if os.path.exists(p):
            out.append(p)
    return out


def _deps():
    deps = [os.path.join(ROOT, "include", "beam_b200.h")]
    for d, _, files in os.walk(CSRC):
        deps += [os.path.join(d, f) for f in files if f.endswith((".cu", ".cuh", ".cpp", ".h"))]
    return deps


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force=False, verbose=False, extra=()):
    if not force and up_to_date():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    objs = []
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"),
              "-I", CSRC]
    for src in _sources():
        obj = os.path.join(OUT_DIR, os.path.basename(src).rsplit(".", 1)[0] + ".o")
        cmd = [NVCC, *common, *ARCH, "-lineinfo", "--expt-relaxed-constexpr", *extra, "-c", src,
               "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-lcuda", "-lcublasLt"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=tuple(a for a in sys.argv[1:] if a.startswith("-X")))
