"""Build libosm_b200.so for sm_100a in-tree (nvcc cross-compiles without a GPU)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(HERE, "libosm_b200.so")

SOURCES = ["osm_capi.cu", "osm_kernels.cu", "osm_router.cu", "osm_experts.cu", "osm_gemv.cu",
           "osm_prefill.cu", "osm_tc.cu", "osm_tcd.cu", "osm_ep.cu"]
HEADERS = ["osm_common.cuh", "osm_kernels.cuh", "osm_tcgen05.cuh"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def build(force: bool = False, verbose: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "osm_b200.h")]
    if force or _stale(LIB, deps):
        cmd = [nvcc()] + NVCC_FLAGS + ["-o", LIB] + srcs
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
