"""Builds libindecis_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

The library links the CUDA runtime statically and resolves the driver's
tensor-map encoder at run time, so it carries no dependency on torch or on
libcuda at link time. Run ``python -m indecis_b200.build`` or call ``build()``.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libindecis_b200.so")
SOURCES = ["libindecis_b200.cu", "spans.cpp", "batcher.cpp"]
HEADERS = ["common.cuh", "exactmath.cuh", "internal.h", "gemm_i8.cu", "gemm_persist.cu", "gemm_pair.cu", "rows_fast.cu", "rows.cu", "rows_ln.cu", "attention.cu", "attention_tc.cu", "attention_short.cu", "siglip.cu", "encoder_f32.cu", "capi.cu", "multi.cu", "siglip_capi.cu", "spans_device.cu", "noalloc.cu", "selfcheck.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-rdc=false",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, extra: list[str] | None = None) -> str:
    """Compiles every .cu into objects, then links the shared library."""
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    inc = [os.path.join(ROOT, "include"), CSRC]
    header_paths = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "indecis_b200.h")]
    objs = []
    for src in SOURCES:
        sp = os.path.join(CSRC, src)
        op = os.path.join(objdir, os.path.splitext(src)[0] + ".o")
        objs.append(op)
        if force or _stale(op, [sp] + header_paths):
            cmd = [_nvcc(), *NVCC_FLAGS, *(extra or []), *[f"-I{i}" for i in inc], "-c", sp, "-o", op]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
               "-o", LIB, *objs, "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv,
          extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
