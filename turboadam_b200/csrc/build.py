"""Build libturboadam_b200.so (sm_100a) in-tree.

    python -m turboadam_b200.csrc.build [--verbose-ptxas]

Flags that make the device arithmetic bit-identical to the host checker:
--fmad=false (no a*b+c contraction; the sources call __fmaf_rn explicitly
where torch fuses), IEEE division and square root, no flush-to-zero.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
OUT = os.path.join(PKG, "libturboadam_b200.so")
SOURCES = [os.path.join(HERE, "ta_api.cu")]
DEPS = SOURCES + [os.path.join(HERE, f) for f in
                  ("ta_kernels.cuh", "ta_codec.cuh", "ta_device.cuh", "ta_math.h")] + [
    os.path.join(os.path.dirname(PKG), "include", "turboadam_b200.h")]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def flags(ptxas_verbose: bool = False) -> list[str]:
    f = [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "--fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
        "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
        "-shared", "-cudart", "static",
    ]
    if ptxas_verbose:
        f += ["-Xptxas", "-v"]
    return f


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(d) <= t for d in DEPS)


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc()] + flags(ptxas_verbose) + ["-o", tmp] + SOURCES
    if not quiet:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(force=a.force or a.verbose_ptxas, ptxas_verbose=a.verbose_ptxas)
    sys.exit(0)
