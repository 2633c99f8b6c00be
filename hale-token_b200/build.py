"""Build recipe for libhale_cuda.so (the product library).

nvcc compiles the CUDA sources for sm_100a only and links them into an
in-tree shared library next to this file, so the .so travels with the
repository snapshot. Flags that keep the arithmetic exact: no fast-math,
--fmad=false (the kernels also use explicit __fmul_rn/__fadd_rn), and the
host side of hale_expf built with -ffp-contract=off.

Usage: python "hale-token_b200/build.py" [--force] [--verbose]
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libhale_cuda.so")
SOURCES = [os.path.join(CSRC, "hale_cuda.cu")]
DEPS = SOURCES + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))] + [
    os.path.join(ROOT, "include", "hale_cuda.h"), os.path.abspath(__file__)]

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--fmad=false",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
    "-shared", "-cudart", "static", "-ldl",
]


def stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(p) > t for p in DEPS)


def build(force=False, verbose=False):
    if not force and not stale():
        return OUT
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, *NVCC_FLAGS, *( ["-Xptxas", "-v"] if verbose else []), *SOURCES, "-o", OUT + ".tmp"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
