"""Build libvxg.so (the sm_100a kernels + C ABI) in-tree with nvcc.

nvcc cross-compiles for sm_100a without a GPU. Flags that matter for parity: -fmad=false (no implicit a*b+c
contraction: every fused multiply-add in the kernels is an explicit __fmaf_rn), IEEE division and square root
(the nvcc defaults; never --use_fast_math), no flush-to-zero; host code with -ffp-contract=off and -mfma (explicit
fma() calls compile to the hardware instruction, which rounds once, as the device's does).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libvxg.so")
ROOT = os.path.dirname(HERE)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
    "-Xcompiler", "-fPIC,-O2,-ffp-contract=off,-mfma",
    "-Xptxas", "-warn-spills",
]


def sources():
    gen = os.path.join(CSRC, "crmath_gen.cpp")  # table generator (a program), not part of the library
    return sorted(f for f in glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")) if f != gen)


def deps():
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(ROOT, "include", "vxg.h")]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in deps())


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.exists(c) or c == "nvcc"):
            return c
    return "nvcc"


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    jobs = []
    for src in sources():
        obj = os.path.join(build_dir, os.path.basename(src) + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        jobs.append((cmd, obj))
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for r in list(ex.map(lambda j: subprocess.run(j[0], check=False), jobs)):
            if r.returncode != 0:
                raise subprocess.CalledProcessError(r.returncode, r.args)
    objs = [o for _, o in jobs]
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC", "-o", LIB, *objs]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
