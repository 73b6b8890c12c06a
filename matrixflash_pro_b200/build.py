"""Build recipe for libmfb.so (sm_100a) — compiled in-tree so it travels with the tree.

    python -m matrixflash_pro_b200.build          # or matrixflash_pro_b200.build.build()

nvcc cross-compiles for sm_100a without a GPU. The library links the CUDA runtime
statically and resolves the driver's cuTensorMapEncodeTiled at run time, so it
needs no libcuda at link time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmfb.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2",
              "-Xcompiler", "-fvisibility=hidden", "-cudart", "static"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h")))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(ROOT, "include", "mfb.h")]
    return all(os.path.getmtime(s) <= t for s in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *(extra_flags or []), "-I", os.path.join(ROOT, "include"),
           "-shared", "-o", LIB + ".tmp", os.path.join(CSRC, "libmfb.cu"), "-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB)
