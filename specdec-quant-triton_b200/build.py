"""Build libspecq.so (the sm_100a kernels behind the C ABI of include/specq.h) in-tree.

    python specdec-quant-triton_b200/build.py [--verbose-ptxas] [--force]

nvcc cross-compiles for sm_100a without a GPU.  The library links the CUDA runtime
statically and reaches the driver only through cudaGetDriverEntryPoint, so it loads on a
machine without a GPU driver (the CPU tests check that every declared symbol is exported).
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO, "include")
OUT = os.path.join(PKG_DIR, "specq", "libspecq.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  glob.glob(os.path.join(INCLUDE, "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = False, trace: bool = False) -> str:
    """Build libspecq.so; trace=True builds libspecq_trace.so with the pipeline trace points."""
    out = OUT.replace("libspecq.so", "libspecq_trace.so") if trace else OUT
    if not force and not trace and up_to_date():
        return OUT
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC]
    if trace:
        cmd += ["-DSPECQ_TRACE"]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, "specq_api.cu"), "-o", out + ".tmp"]
    if not quiet:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libspecq.so")
    if verbose_ptxas or not quiet:
        sys.stderr.write(res.stderr)
    os.replace(out + ".tmp", out)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--trace", action="store_true", help="also build libspecq_trace.so (-DSPECQ_TRACE)")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))
    if args.trace:
        print(build(force=True, trace=True))


if __name__ == "__main__":
    main()
