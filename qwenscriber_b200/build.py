"""Builds libqwenscriber_cuda.so in-tree for sm_100a (B200).

nvcc compiles every .cu and .cpp under csrc/ with
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` and links one shared
library next to this file. Objects go to ``_build/`` (git-ignored). Rebuilds
only what changed (by modification time).
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libqwenscriber_cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
CUDA_INC = os.path.join(os.path.dirname(os.path.dirname(NVCC)), "include")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", CSRC, "-I", INCLUDE]


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "qwenscriber_cuda.h"))
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))
    headers = _headers()
    objects = []
    for src in sources:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objects.append(obj)
        # A source may include another (qwc_decode_wide.cu compiles qwc_decode.cu
        # with a wider weight ring), so every source counts as a dependency.
        deps = [path, *headers, *(os.path.join(CSRC, f) for f in sources if f.endswith(".cu")), __file__]
        if not _stale(obj, deps) and not ptxas_verbose:
            continue
        cmd = [NVCC, *ARCH, *COMMON, "-c", path, "-o", obj]
        if src.endswith(".cpp"):
            cmd = [CXX, "-O3", "-std=c++17", "-fPIC", "-Wall", "-I", CSRC, "-I", INCLUDE, "-I", CUDA_INC,
                   "-c", path, "-o", obj]
        elif ptxas_verbose:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if _stale(LIB, objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objects, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv)
