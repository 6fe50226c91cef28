"""Build libdsca_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m dsca_moe_b200.build          # or __graft_entry__.build()

Objects go to dsca_moe_b200/_build/, the library to dsca_moe_b200/lib/libdsca_b200.so.
cudart is linked statically, so the library does not depend on the CUDA runtime that the
host process (PyTorch) loaded.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libdsca_b200.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = shutil.which("nvcc") or os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I" + INCLUDE] + ARCH
CU_SOURCES = ["router.cu", "router_tc.cu", "dispatch.cu", "gemm_sm100.cu", "gemm_sm100_pair.cu", "gemm_sm100_fp8.cu", "gemm_sm100_fp8t.cu", "gemm_simt.cu", "abi.cu",
              "ffn_static_scratch.cu", "ep.cu", "qos.cu"]
CXX_SOURCES = ["plan.cpp"]


def _newer(src_list, target):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_list)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    # every header of the package (a change to any of them rebuilds every object)
    headers = sorted(os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h")))
    headers.append(os.path.join(INCLUDE, "dsca_b200.h"))
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if _newer([s] + headers, o) or ptxas_verbose:
            cmd = [NVCC, "-c", s, "-o", o] + NVCC_FLAGS
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    for src in CXX_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if _newer([s] + headers, o):
            cmd = ["g++", "-O2", "-fPIC", "-std=c++17", "-I" + INCLUDE, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if _newer(objs, LIB):
        cmd = [NVCC, "-shared", "-o", LIB] + objs + ARCH + ["-cudart", "static", "-Xcompiler", "-fPIC"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_verbose="-v" in sys.argv))
