"""Build recipe for libb200linear.so (the product library) with nvcc.

Compiles every CUDA source in csrc/ for sm_100a and links them, together
with the C++ adapter that implements the reference engine's
infer::cuda Linear functions on top of the C ABI, into one shared library
placed next to this file.  Object files are rebuilt only when a source or
header is newer.  Usable as ``python build.py`` or via ``build()``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libb200linear.so")
INCLUDE = os.path.join(REPO, "include")

SOURCES = ["gemv.cu", "gemv_i8tc.cu", "gemm_simt.cu", "gemm_sm100.cu", "gemm_w8t.cu", "capi.cu", "noalloc.cu", "attention_tc.cu", "engine.cu",
           "decode_persistent.cu",
           "sharded.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    out = [os.path.join(INCLUDE, "b200_linear.h"), os.path.join(INCLUDE, "b200_engine.h")]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return out


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, extra=()) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    with ThreadPoolExecutor(max_workers=min(4, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-o", LIB, *objs,
               "-lnccl"]
        subprocess.run(cmd, check=True)
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
