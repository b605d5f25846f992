"""Build libprismkv_b200.so in-tree with nvcc for sm_100a.

``python -m prismkv_b200.build`` (or ``build()``) compiles csrc/pkv_lib.cu
into prismkv_b200/libprismkv_b200.so.  The library statically links the CUDA
runtime, takes streams from the caller and exports only the C ABI declared in
include/prismkv_b200.h.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libprismkv_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-shared", "-cudart", "static",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the PrismKV B200 library needs the CUDA toolkit to build")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    csrc = os.path.join(HERE, "csrc")
    deps = [os.path.join(csrc, s) for s in os.listdir(csrc) if s.endswith((".cu", ".cuh"))]
    deps.append(os.path.join(ROOT, "include", "prismkv_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"),
           os.path.join(HERE, "csrc", "pkv_lib.cu"), "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
