"""Builds the in-tree shared library kokopop_b200/libkokopop_b200.so for
sm_100a with nvcc (no JIT cache: the .so travels with the tree).

    python -m kokopop_b200.build
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libkokopop_b200.so")

CU_SOURCES = ["kk_kernels.cu", "kk_conv_simt.cu", "kk_conv_tc.cu", "kk_istft_static.cu", "kk_lstm.cu", "kk_frontend.cu",
              "kk_vocos.cu"]
CXX_SOURCES = ["kk_host.cpp", "kk_queue.cpp", "kk_stream.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"] + ARCH


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(HERE, "..", "include", "kokopop_b200.h"))
    objs = []
    nv = nvcc()
    for src in CU_SOURCES + CXX_SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objs.append(obj)
        if not _stale(obj, [path] + headers) and not ptxas_info:
            continue
        cmd = [nv] + NVCC_FLAGS + ["-c", path, "-o", obj]
        if src.endswith(".cpp"):
            cmd = [nv, "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-x", "cu"] + ARCH + ["-c", path, "-o", obj]
        if ptxas_info and src.endswith(".cu"):
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        cmd = [nv, "-shared"] + ARCH + objs + ["-o", LIB, "-lcudart"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="--ptxas" in sys.argv))
