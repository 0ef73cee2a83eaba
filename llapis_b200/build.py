"""Builds libmoeb200.so in-tree (llapis_b200/lib/) with nvcc for sm_100a.

    python -m llapis_b200.build [--force]

Device code is one translation unit (csrc/kernels.cu); the C-ABI host side (csrc/api.cpp) and the
weight quantiser (csrc/quant.cpp) are plain C++ built with -ffp-contract=off so their float code
rounds exactly as written (the quantiser's bytes must equal the reference quantiser's).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libmoeb200.so")
INCLUDE = os.path.join(ROOT, "include")

SOURCES = ["kernels.cu", "api.cpp", "quant.cpp", "store.cpp", "load.cpp"]
HEADERS = ["common.cuh", "params.h", "ggml_tables.inc", "prefill.cuh", "gateup_lx.cuh", "mid.cuh"]
PUBLIC_HEADERS = ["moeb200.h", "moert_cuda.h", "moert_store.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST_FLAGS = "-fPIC,-O2,-ffp-contract=off,-mf16c,-mavx2,-mfma,-pthread"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the library builds only with the CUDA toolkit (no CPU fallback)")


def _fingerprint() -> str:
    h = hashlib.sha256()
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, f) for f in PUBLIC_HEADERS]
    for f in files:
        if os.path.exists(f):
            with open(f, "rb") as fh:
                h.update(fh.read())
    h.update(" ".join(ARCH + [HOST_FLAGS]).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if its sources changed; returns the path of the .so."""
    os.makedirs(LIBDIR, exist_ok=True)
    stamp = os.path.join(LIBDIR, ".fingerprint")
    fp = _fingerprint()
    if not force and os.path.exists(LIB) and os.path.exists(stamp) and open(stamp).read() == fp:
        return LIB
    nvcc = _nvcc()
    objs = []
    for src in SOURCES:
        obj = os.path.join(LIBDIR, src + ".o")
        cmd = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", HOST_FLAGS,
               "-I", CSRC, "-I", INCLUDE, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart", "-Xcompiler", "-pthread"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    with open(stamp, "w") as fh:
        fh.write(fp)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
