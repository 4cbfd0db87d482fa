"""Build the in-tree native artefacts.

    libmidgecuda.so   sm_100a kernels + C ABI (include/midgecuda.h)
    bin/midged        the C host: midged's protocol loop over the C ABI

Both land inside the package directory so they travel with the source tree
(no site-packages install, no JIT cache).  Run: python -m midge_b200.build
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libmidgecuda.so")
MIDGED = os.path.join(PKG, "bin", "midged")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
GCC = "/usr/bin/gcc"

CU_SOURCES = ["mg_abi.cu", "mg_gemv.cu", "mg_moe.cu", "mg_attn.cu", "mg_model.cu", "mg_stream.cu", "mg_gemm.cu", "mg_prefill.cu", "mg_noalloc.cu", "mg_ep.cu", "mg_ep_xchg.cu", "mg_sample.cu", "mg_selftest.cu", "mg_bsmoe.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd, cwd=None):
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd))
    return r.stdout + r.stderr


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(force=False, verbose=False):
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(INCLUDE, "midgecuda.h"))
    if not force and not _stale(LIB, deps):
        return LIB
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for s in srcs:
        o = os.path.join(objdir, os.path.basename(s) + ".o")
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC,
               "-c", s, "-o", o]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        out = _run(cmd)
        if verbose and out:
            sys.stderr.write(out)
        objs.append(o)
    _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-lrt", "-lpthread", "-ldl"])
    return LIB


def build_midged(force=False):
    srcs = [os.path.join(HOST, f) for f in ("midged.c",)]
    deps = srcs + [os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith(".h")] + [LIB]
    if not os.path.exists(srcs[0]):
        return None
    if not force and not _stale(MIDGED, deps):
        return MIDGED
    os.makedirs(os.path.dirname(MIDGED), exist_ok=True)
    _run([GCC, "-O2", "-std=c11", "-D_GNU_SOURCE", "-Wall", "-Wno-unused-function", "-I", INCLUDE, "-I", HOST,
          *srcs, "-o", MIDGED, "-L", PKG, "-lmidgecuda", "-Wl,-rpath,$ORIGIN/..", "-lm"])
    return MIDGED


def build_all(force=False, verbose=False):
    build_lib(force=force, verbose=verbose)
    build_midged(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
