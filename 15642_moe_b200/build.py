"""Build recipe for the native libraries of this package (in-tree, no JIT cache).

* ``libmoe_b200.so``     - every CUDA kernel and the C ABI of ``include/moe_b200.h``,
  compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) without
  fast-math: the router's sigmoid, the SwiGLU exponential and the scale divisions must be
  the IEEE-rounded operations the CPU checker restates.
* ``libmoe_synth_cpu.so`` - the CPU twin of the seeded input generator (plain C, OpenMP,
  no FMA contraction so its fp32 arithmetic matches the GPU generator bit for bit).

Run ``python -m 15642_moe_b200.build`` from the repository root, or call :func:`build_all`.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")

CUDA_LIB = os.path.join(PKG_DIR, "libmoe_b200.so")
SYNTH_CPU_LIB = os.path.join(PKG_DIR, "libmoe_synth_cpu.so")

CUDA_SOURCES = ["moe_b200.cu"]
CUDA_HEADERS = ["moe_common.cuh", "route.cuh", "ep.cuh", "gemm1.cuh", "gemm2.cuh", "pack.cuh", "quant.cuh", "gate.cuh", "synth.cuh",
                "synth_core.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmoe_b200.so")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    deps = [os.path.join(CSRC, f) for f in CUDA_SOURCES + CUDA_HEADERS]
    deps.append(os.path.join(INCLUDE, "moe_b200.h"))
    if not force and not _stale(CUDA_LIB, deps):
        return CUDA_LIB
    tmp = CUDA_LIB + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-Xptxas", "-v",
           "-o", tmp, os.path.join(CSRC, "moe_b200.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_synth_cpu(force: bool = False) -> str:
    src = os.path.join(CSRC, "synth_cpu.c")
    deps = [src, os.path.join(CSRC, "synth_core.h")]
    if not force and not _stale(SYNTH_CPU_LIB, deps):
        return SYNTH_CPU_LIB
    tmp = SYNTH_CPU_LIB + ".tmp"
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-I", CSRC, "-o", tmp, src, "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("gcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    os.replace(tmp, SYNTH_CPU_LIB)
    return SYNTH_CPU_LIB


def build_all(force: bool = False, verbose: bool = False) -> list[str]:
    return [build_cuda(force, verbose), build_synth_cpu(force)]


if __name__ == "__main__":
    for path in build_all(force="--force" in sys.argv, verbose="-v" in sys.argv):
        print(path)
