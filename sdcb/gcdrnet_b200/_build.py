"""Builds libgcdr_cuda.so in-tree with nvcc for sm_100a (B200).

The library is the product: hand-written sm_100a kernels (tcgen05 implicit-GEMM
convolutions, fp32 stem/head, token kernels), the C++ worker/enhancer and the C
ABI of include/gcdr_cuda.h.  It links the CUDA runtime statically and loads
the driver's tensor-map encoder at run time, so it needs no libcuda at link
time and builds on a machine without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(PKG, "csrc")
ROOT = os.path.dirname(os.path.dirname(PKG))
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libgcdr_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", SRC, "-I", INCLUDE]

SOURCES = ["model.cpp", "conv_tc.cu", "conv_rw.cu", "conv_ref.cu", "kernels.cu", "pipeline.cu", "capi.cu", "noalloc.cu"]


def _headers():
    hs = [os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "gcdr_cuda.h"))
    return hs


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    newest = max(os.path.getmtime(h) for h in _headers() + [src])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    if src.endswith(".cpp"):
        cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-fvisibility=hidden", "-I", SRC, "-I", INCLUDE,
               "-I", "/usr/local/cuda/include", "-c", src, "-o", obj]
    else:
        cmd = [NVCC] + ARCH + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = [os.path.join(SRC, s) for s in SOURCES]
    if force:
        for s in srcs:
            o = os.path.join(OBJ, os.path.basename(s) + ".o")
            if os.path.exists(o):
                os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    tmp = LIB + ".tmp%d" % os.getpid()
    cmd = [NVCC] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
