"""Build the sm_100a CUDA library (talos_b200/_lib/libtalos_cuda.so) and the
synthetic-model generator (talos_b200/_lib/libtalos_synth.so) in-tree.

    python -m talos_b200.build [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
SYNTH = os.path.join(PKG, "synth")
OUT = os.path.join(PKG, "_lib")
CUDA_LIB = os.path.join(OUT, "libtalos_cuda.so")
SYNTH_LIB = os.path.join(OUT, "libtalos_synth.so")

CU_SOURCES = ["kernels.cu", "matvec.cu", "gemm.cu", "runtime.cu"]
CU_DEPS = CU_SOURCES + ["common.cuh", "kernels.cuh", "ptx.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fno-fast-math",
    "--expt-relaxed-constexpr",
    "-shared",
]


# NCCL (opened with dlopen at run time) bootstraps tensor-parallel contexts;
# only its header is needed here. The all-reduce runs inside the per-token kernel.
LINK = ["-ldl", "-Xlinker", "--no-undefined"]  # a missing definition fails the build, not the first load


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    deps = [os.path.join(CSRC, f) for f in CU_DEPS] + [os.path.join(ROOT, "include", "talos_cuda.h")]
    if not force and not _newer(CUDA_LIB, deps):
        return CUDA_LIB
    os.makedirs(OUT, exist_ok=True)
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", CUDA_LIB + ".tmp",
           *[os.path.join(CSRC, f) for f in CU_SOURCES], *LINK]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(CUDA_LIB + ".tmp", CUDA_LIB)
    return CUDA_LIB


def build_synth(force: bool = False) -> str:
    src = os.path.join(SYNTH, "synth.c")
    if not force and not _newer(SYNTH_LIB, [src]):
        return SYNTH_LIB
    os.makedirs(OUT, exist_ok=True)
    cmd = ["gcc", "-O2", "-std=gnu11", "-fPIC", "-shared", "-pthread", "-ffp-contract=off",
           "-o", SYNTH_LIB + ".tmp", src, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(SYNTH_LIB + ".tmp", SYNTH_LIB)
    return SYNTH_LIB


def build(force: bool = False, verbose: bool = False) -> None:
    build_cuda(force, verbose)
    build_synth(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
