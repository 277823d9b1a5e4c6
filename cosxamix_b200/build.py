"""Build recipe of cosxamix_b200/libcxm.so (sm_100a), in-tree.

    python -m cosxamix_b200.build          # or __graft_entry__.build()

Host C++ (GGUF reader, synthetic-model writer) is compiled by g++ without FMA
contraction (the k-quant writers must round exactly as the reference's Rust);
the CUDA sources by nvcc for sm_100a only.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libcxm.so")
BUILD = os.path.join(os.path.dirname(HERE), "_build")

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXX_FLAGS = ["-O3", "-fPIC", "-std=c++17", "-ffp-contract=off", "-Wall", "-Wno-unused-function"]
CUDA_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off",
                     "--expt-relaxed-constexpr", "-Xptxas", "-O3"]

CXX_SOURCES = ["gguf.cpp", "synth.cpp"]
CU_SOURCES = ["model.cu"]
HEADERS = sorted(f for f in os.listdir(CSRC) if f.endswith((".h", ".cuh")))


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd))


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(os.path.dirname(HERE), "include", "cxm.h")]
    objs = []
    for src in CXX_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if _newer(o, [s] + hdrs):
            _run(["g++", *CXX_FLAGS, "-c", s, "-o", o])
        objs.append(o)
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if _newer(o, [s] + hdrs) or ptxas_info:
            cmd = [NVCC, *CUDA_FLAGS, "-c", s, "-o", o]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
                r = subprocess.run(cmd, capture_output=True, text=True)
                sys.stdout.write(r.stderr)
                if r.returncode:
                    raise RuntimeError("nvcc failed")
            else:
                _run(cmd)
        objs.append(o)
    if _newer(OUT, objs):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", OUT, *objs, "-lpthread"])
    if verbose:
        print("built", OUT)
    return OUT


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
