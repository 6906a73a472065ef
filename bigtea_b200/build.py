"""Build recipe for libbigtea_decode.so (sm_100a) -- the one compiled artefact of the package.

The library is built in-tree (bigtea_b200/libbigtea_decode.so) with nvcc for
`-gencode arch=compute_100a,code=sm_100a`. `--fmad=false` and `-ffp-contract=off` keep every
multiply and add separately rounded unless the source writes fmaf: the decode layer's
arithmetic contract depends on it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libbigtea_decode.so")
SOURCES = ["kernels.cu", "step_kernel.cu", "expert_stream.cu", "xcache.cu", "mma.cu", "sampler.cu", "engine.cu"]
DEPS = SOURCES + ["kernels.cuh", "kquant.cuh", "bt_common.cuh", "stage.cuh", "step_kernel.cuh", "expert_stream.cuh", "xcache_dev.cuh", "umma.cuh", "sampler.cuh",
                  "expert_cache.h"]
HEADER = os.path.join(os.path.dirname(PKG), "include", "bigtea_decode.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "--fmad=false", "-std=c++17",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fopenmp",
    "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libbigtea_decode.so")


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    paths = [os.path.join(CSRC, f) for f in DEPS] + [HEADER]
    return any(os.path.getmtime(p) > t for p in paths)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-o", LIB + ".tmp", *[os.path.join(CSRC, f) for f in SOURCES], "-lgomp"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
