"""Builds librwgpu.so in-tree for sm_100a with nvcc.

The library links NCCL from the same wheel torch loads (nvidia/nccl in site-packages),
so a process that imports torch and this library shares one libnccl.so.2.
Run as `python rustwood_b200/build.py` (a plain script: importing the package would
load the library it is about to rebuild) or load this file and call build().
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "librwgpu.so")
SOURCES = ["rwgpu.cu", "train_kernels.cu", "predict_kernels.cu", "noalloc.cu", "peer_kernels.cu",
           "boundaries.cu", "encode.cu"]
HEADERS = ["rw_internal.cuh", "rw_expf.h", os.path.join("..", "..", "include", "rwgpu.h")]


def nccl_paths() -> tuple[str, str]:
    """Include and lib dirs of the NCCL wheel torch uses; falls back to /usr."""
    purelib = sysconfig.get_paths()["purelib"]
    base = os.path.join(purelib, "nvidia", "nccl")
    inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
        return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [__file__]
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def nvcc_command() -> list[str]:
    inc, lib = nccl_paths()
    return [
        nvcc(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-lineinfo", "-O3", "-std=c++17",
        # Bit-exact f32/f64 arithmetic shared with the CPU restatement: no FMA contraction.
        "--fmad=false",
        "-Xcompiler", "-fPIC,-ffp-contract=off,-O2",
        "-shared", "-o", LIB,
        *[os.path.join(CSRC, s) for s in SOURCES],
        f"-I{inc}", f"-L{lib}", "-l:libnccl.so.2",
        "-Xlinker", f"-rpath,{lib}",
    ]


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = nvcc_command()
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
