"""Builds the in-tree CUDA library ``hybridagent_b200/lib/libhybridagent_b200.so`` for sm_100a.

    python -m hybridagent_b200.build [--force]

nvcc compiles the kernels for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``),
with ``-fmad=false`` (every fused multiply-add in the kernels is an explicit ``__fmaf_rn``)
and the host compiler at ``-ffp-contract=off`` (the host computes the step's fp32 scalars in
double exactly as CPython does).  The CUDA runtime is linked statically; NCCL is opened at
run time (``comm.cpp``).  The library is rebuilt only when a source is newer than it.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ_DIR = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libhybridagent_b200.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["adamw.cu", "gradnorm.cu", "gather.cu", "p2p.cu"]
CPP_SOURCES = ["host.cpp", "comm.cpp"]


def _nccl_include() -> str:
    cand = os.path.join(sysconfig.get_paths()["purelib"], "nvidia", "nccl", "include")
    if os.path.exists(os.path.join(cand, "nccl.h")):
        return cand
    return "/usr/include"


def _sources() -> list[str]:
    files = [os.path.join(CSRC, f) for f in CU_SOURCES + CPP_SOURCES]
    files += [os.path.join(CSRC, "ha_common.cuh"), os.path.join(CSRC, "ha_nvtx.h"),
              os.path.join(INCLUDE, "hybridagent_b200.h"), __file__]
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _sources())


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile every source and link the shared library; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    objs = []
    for src in CU_SOURCES:
        obj = os.path.join(OBJ_DIR, src + ".o")
        cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC,-ffp-contract=off",
               "-I", INCLUDE, "-c", os.path.join(CSRC, src), "-o", obj]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd, verbose)
        objs.append(obj)
    for src in CPP_SOURCES:
        obj = os.path.join(OBJ_DIR, src + ".o")
        _run([NVCC, "-x", "c++", "-O2", "-std=c++17", "-Wno-deprecated-gpu-targets", "-Xcompiler", "-fPIC,-ffp-contract=off,-Wall", "-I", INCLUDE,
              "-I", _nccl_include(), "-c", os.path.join(CSRC, src), "-o", obj], verbose)
        objs.append(obj)
    # export the C ABI (ha_*) only: the static CUDA runtime and internal C++ stay local
    exports = os.path.join(OBJ_DIR, "exports.map")
    with open(exports, "w") as f:
        f.write("{ global: ha_*; local: *; };\n")
    tmp = LIB_PATH + ".tmp"
    _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-ldl", "-lrt", "-lpthread",
          "-Xlinker", f"--version-script={exports}"], verbose)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv))
