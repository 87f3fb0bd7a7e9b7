"""Build recipe for the sm_100a shared library ``libmoe_fp8_ds.so``.

The library is compiled in-tree (next to this file) with nvcc for
``arch=compute_100a,code=sm_100a`` only; nvcc cross-compiles without a GPU.
It links the CUDA runtime statically and resolves the driver entry point
``cuTensorMapEncodeTiled`` at run time, so it needs no ``-lcuda``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libmoe_fp8_ds.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
INCLUDE = os.path.join(os.path.dirname(HERE), "include")  # moe_fp8_ds.h, the C ABI
SOURCES = ["moe_route.cu", "moe_gemm.cu", "moe_decode.cu", "moe_quant.cu", "moe_ep.cu", "moe_api.cu", "moe_noalloc.cu"]
HEADERS = ["moe_common.cuh", "moe_kernels.h", "moe_routing.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-I", INCLUDE,
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _inputs() -> list[str]:
    inc = os.path.join(INCLUDE, "moe_fp8_ds.h")
    return [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [inc]


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    nvcc = _nvcc()
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc, *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
