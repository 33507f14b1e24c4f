"""Builds libeahmmf_b200.so in-tree (cross-compiles for sm_100a; no GPU needed).

    python eahmmf_inference_prototype_v-0.1.0_b200/build.py [--force]

The library is plain nvcc output: no torch extension, no JIT cache, so the same .so travels to the
GPU box with the repository. Denormals must stay IEEE (no -use_fast_math / -ftz=true): the K-quant
decoders build exact floats from denormal bit patterns.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libeahmmf_b200.so")
SOURCES = ["kernels.cu", "moe.cu", "capi.cu", "device.cu", "decode.cu", "engine.cu", "gemm.cu", "ep.cu", "sample.cu", "verify.cu"]
HEADERS = ["common.cuh", "kq.cuh", "ksb.cuh", "kernels.cuh", "decode.cuh", "tc.cuh", "sample.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _inputs():
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(os.path.dirname(HERE), "include", "eahmmf_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    objs, procs = [], []
    for src in SOURCES:  # translation units compile in parallel
        obj = os.path.join(CSRC, "_build", src.replace(".cu", ".o"))
        os.makedirs(os.path.dirname(obj), exist_ok=True)
        cmd = [NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((subprocess.Popen(cmd), cmd))
        objs.append(obj)
    for p, cmd in procs:
        if p.wait() != 0:
            raise subprocess.CalledProcessError(p.returncode, cmd)
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static", *objs, "-o", tmp],
                   check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
