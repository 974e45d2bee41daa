"""Build libtextsift_cuda.so in-tree with nvcc for sm_100a (B200).

Usage: python -m textsift_b200.build  (or textsift_b200.build.build()).
The library is self-contained: CUDA runtime linked statically, the driver's
cuTensorMapEncodeTiled resolved at run time, no torch headers.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libtextsift_cuda.so")
SOURCES = ["k_gemm_tc.cu", "k_gemm_tm.cu", "k_simt.cu", "k_router.cu", "k_attn.cu", "k_attn_umma.cu", "k_viterbi.cu", "k_selftest.cu", "runtime.cu", "ep.cu", "noalloc.cu", "onnx_load.cu", "tokenizer.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-I", INCLUDE, "-I", CSRC]


def _newest_input() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, "textsift_cuda.h"), __file__]
    return max(os.path.getmtime(p) for p in paths)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest_input():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-ldl"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
