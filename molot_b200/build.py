"""Builds libmolot_b200.so in-tree with nvcc for sm_100a.

    python -m molot_b200.build [--force] [--ptxas-verbose]

The library is a plain C-ABI shared object (include/molot_b200.h); it links
the CUDA runtime statically, so it needs only the driver at run time.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libmolot_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
    "-Xcudafe", "--diag_suppress=177",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and not shutil.which(cand):
        raise RuntimeError("nvcc not found; set NVCC")
    return cand


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(INCLUDE, "molot_b200.h")]


def up_to_date() -> bool:
    if not os.path.isfile(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in deps())


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = False) -> str:
    if not force and not ptxas_verbose and up_to_date():
        return LIB
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs, cmds = [], []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if not quiet:
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
        objs.append(obj)
    # translation units compile independently: run them side by side
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as ex:
        for f in [ex.submit(subprocess.run, c, check=True) for c in cmds]:
            f.result()
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lpthread"]
    if not quiet:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args(argv)
    build(force=args.force, ptxas_verbose=args.ptxas_verbose)
    return 0


if __name__ == "__main__":
    sys.exit(main())
