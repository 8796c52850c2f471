"""Builds libsarr.so (the sm_100a kernels + C ABI) in place with nvcc.

Usage: python sar-3dgs_b200/build.py [--force] [--verbose]

The device code is compiled with nvcc's default floating-point settings (no
--use_fast_math, FMA contraction on), the same settings under which the
reference module is JIT-built by cuda_rasterizer/__init__.py:51-55; the
tile-list parity depends on it. The host code is compiled for the baseline
x86-64 target (no -march), so that its float math (view setup) rounds like
the reference's host code.
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(HERE, "libsarr.so")
SOURCES = ["sarr_kernels.cu", "sarr_abi.cu", "sarr_static.cu", "sarr_train.cu", "sarr_densify.cu"]
HEADERS = ["sarr_common.cuh", "sarr_internal.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda_home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _inputs():
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(INCLUDE, "sarr.h"))
    files.append(os.path.abspath(__file__))
    return files


def up_to_date(target, inputs):
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(f) <= t for f in inputs)


def build(force=False, verbose=False, ptxas_verbose=False):
    if not force and up_to_date(LIB, _inputs()):
        return LIB
    objs = []
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    common = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
              "-I", INCLUDE, "-I", CSRC]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    for src in SOURCES:
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = common + ["-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose))
    sys.exit(0)
