"""Builds libk3xb.so (all CUDA sources, sm_100a only) into project-k3x_b200/k3xb/.

Used by __graft_entry__.build(); nvcc cross-compiles without a GPU.
"""
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "k3xb")
LIB = os.path.join(OUT_DIR, "libk3xb.so")
OBJ_DIR = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++20", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
                     "--expt-relaxed-constexpr", "-fmad=true", "-I", CSRC,
                     "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, extra=()) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    headers = (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp")) +
               [os.path.join(ROOT, "include", "k3xb.h")])
    objs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, [src] + headers):
            cmd = [nvcc()] + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
