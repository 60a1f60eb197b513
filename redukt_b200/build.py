"""Builds libredukt_gpu.so in-tree for sm_100a (B200).  `python -m redukt_b200.build`."""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libredukt_gpu.so")
SOURCES = ["redukt_gpu.cu"]
HEADERS = ["rk_math.cuh", "rk_kernels.cuh", "rk_fused.cuh", "rk_tc.cuh", "rk_rwkv7.cuh", "rwkv7_engine.cuh", "rk_cdf.cuh", "rk_exp_table.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "--shared",
    "-Xcompiler", "-fPIC,-Wall,-Wno-unused-function",
    "-Xptxas", "-warn-spills",
]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "redukt_gpu.h"))
    return any(os.path.exists(p) and os.path.getmtime(p) > t for p in deps)


ARC_LIB = os.path.join(HERE, "libredukt_archive.so")
ARC_SOURCES = ["rk_archive.cpp"]


def build_archive(force: bool = False) -> str:
    """libredukt_archive.so: the host range coder, CRC-32, container and text workload (C++)."""
    srcs = [os.path.join(CSRC, s) for s in ARC_SOURCES] + [os.path.join(HERE, "..", "include", "redukt_archive.h")]
    if not force and os.path.exists(ARC_LIB) and all(os.path.getmtime(p) <= os.path.getmtime(ARC_LIB) for p in srcs):
        return ARC_LIB
    cxx = os.environ.get("CXX", "g++")
    cmd = [cxx, "-O3", "-std=c++17", "-shared", "-fPIC", "-Wall", "-o", ARC_LIB + ".tmp", srcs[0]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("g++ failed building libredukt_archive.so")
    os.replace(ARC_LIB + ".tmp", ARC_LIB)
    return ARC_LIB


def build(force: bool = False, verbose: bool = False) -> str:
    build_archive(force)
    if not force and not _stale():
        return LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, *NVCC_FLAGS, "-o", LIB + ".tmp", *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(-len(SOURCES) - 2, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libredukt_gpu.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
