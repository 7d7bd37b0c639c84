"""Builds libgpt_b200.so in-tree (cutilegpt_b200/lib/) with nvcc for sm_100a.

The library is one translation unit (libgpt_b200.cu) linked against the
static CUDA runtime, so it loads on machines without a GPU driver (tests
check the exported symbols there) and carries no libcudart dependency.
The driver API entry point it needs (cuTensorMapEncodeTiled) is resolved
at run time through cudaGetDriverEntryPoint.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgpt_b200.so")
SOURCES = ["libgpt_b200.cu", "common.cuh", "capi.cu", "elementwise.cu", "gemm_tc.cu", "gemm_skinny.cu", "gemm_rows.cu",
           "gemm_simt.cu", "attention_tc.cu", "attention.cu", "decode.cu", "decode_noalloc.cu",
           "sampling.cu"]
HEADER = os.path.join(os.path.dirname(PKG), "include", "gpt_b200.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
    "-shared",
]


def nvcc_path():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(HERE, s) for s in SOURCES] + [HEADER, __file__]
    return all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, extra=()):
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, *extra, "-o", tmp, os.path.join(HERE, "libgpt_b200.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=HERE)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    args = sys.argv[1:]
    extra = []
    if "--ptxas-v" in args:
        extra += ["-Xptxas", "-v"]
    print(build(force=True, verbose=True, extra=extra))
