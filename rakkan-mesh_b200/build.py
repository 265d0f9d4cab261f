"""Builds librakkan_cuda.so (the CUDA backend) in-tree for sm_100a.

Usage: python rakkan-mesh_b200/build.py [--force]

Float flags: -fmad=false (no product fused into an FMA, device code) and
-ffp-contract=off (the same for host code), -ftz=false (denormals kept),
-prec-div/-prec-sqrt=true: the kernels reproduce the reference CPU path's
bits only with IEEE single roundings everywhere.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "librakkan_cuda.so")
SOURCES = ["rk_matvec.cu", "rk_layer.cu", "rk_tensor.cu", "rk_gen.cu", "rk_capi.cu", "rk_noalloc.cu", "rk_mvmany.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-fmad=false", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
    "-Xptxas", "-v" if os.environ.get("RK_PTXAS_VERBOSE") else "-O3",
]


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh"))]
    files.append(os.path.join(HERE, "..", "include", "rakkan_cuda.h"))
    files.append(os.path.abspath(__file__))
    return files


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs, cmds = [], []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmds.append([NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj])
        objs.append(obj)

    def compile_one(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)

    # The translation units compile independently, so in parallel.
    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as ex:
        list(ex.map(compile_one, cmds))
    tmp = LIB + ".tmp"
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", tmp]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
