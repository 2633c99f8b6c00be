"""Build recipe for the CPU oracle (test infrastructure, not the product).

Compiles oracle/hale_oracle.c into oracle/_build/libhale_oracle.so with the
flags that keep it bit-faithful to the Rust reference: no FMA contraction and
no fast-math. A second copy built with -march=native is what bench.py's CPU
baseline may time; the tests always use the portable one.

Usage: python oracle/build.py [--force]
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
SRC = os.path.join(HERE, "hale_oracle.c")
HDR = os.path.join(HERE, "hale_oracle.h")

VARIANTS = {
    "libhale_oracle.so": [],
    "libhale_oracle_native.so": ["-march=native"],
}


def _stale(out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(p) > t for p in (SRC, HDR, __file__))


def build(force=False, variants=None):
    os.makedirs(BUILD, exist_ok=True)
    outs = []
    for name, extra in VARIANTS.items():
        if variants is not None and name not in variants:
            continue
        out = os.path.join(BUILD, name)
        if force or _stale(out):
            cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC",
                   "-shared", "-std=c11", "-Wall", *extra, SRC, "-o", out + ".tmp", "-lm"]
            subprocess.run(cmd, check=True)
            os.replace(out + ".tmp", out)
        outs.append(out)
    return outs


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv):
        print(p)
