"""Build librw4.so, the RW4 C-ABI library, for sm_100a with nvcc (in-tree, no JIT cache).

    python -m rocketllm_b200.csrc.build          # or: python rocketllm_b200/csrc/build.py

Every .cu / .cpp file in this folder is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into
``rocketllm_b200/librw4.so`` next to the package, so the library travels with the source tree.
Rebuilds only when a source or header is newer than the library.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "librw4.so")
BUILD_DIR = os.path.join(PKG, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def sources():
    return sorted(glob.glob(os.path.join(HERE, "*.cu")) + glob.glob(os.path.join(HERE, "*.cpp")))


def headers():
    return (glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(HERE, "*.h"))
            + glob.glob(os.path.join(ROOT, "include", "*.h")))


def stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, force=False, extra=()):
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    hdrs = headers()
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if not force and not stale(obj, [src] + hdrs):
            continue
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
               "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj, *extra]
        if src.endswith(".cpp"):
            cmd[1:1] = ["-x", "cu"]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcuda", "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
