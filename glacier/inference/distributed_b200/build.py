"""Build libglacier_b200.so (sm_100a) in-tree with nvcc.

Usage: python -m glacier.inference.distributed_b200.build [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libglacier_b200.so")
REPO = os.path.abspath(os.path.join(HERE, "..", "..", ".."))
INCLUDE = os.path.join(REPO, "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off",
          "-I", CSRC, "-I", INCLUDE, "--expt-relaxed-constexpr"]
SOURCES = ["api.cu", "gemv_q4k.cu", "gemv_chain.cu", "decode_fused.cu", "decode_wide.cu", "router.cu", "wire.cu", "prefill.cu", "grouped_mma.cu",
           "noalloc.cu", "ep.cu", "comm.cu", "attention.cu", "stage.cu", "synth.cpp"]
HEADERS = ["common.cuh", "gemv_lane.cuh", "kernels.h", "synth.h"]


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "glacier_b200.h")]
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC, *ARCH, *COMMON, *os.environ.get("GLC_NVCC_DEFINES", "").split(), "-c", path, "-o", obj]
    if os.environ.get("GLC_PTXAS_VERBOSE") and src.endswith(".cu"):
        cmd.insert(1, "-Xptxas=-v")
    subprocess.check_call(cmd)
    return obj


def build(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        subprocess.check_call([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-ldl"])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
