"""Build the sm_100a shared library ``libqb.so`` in-tree with nvcc.

    python -m hackthenorth_b200.build [--force] [--verbose]

The library is the product's only compute path; ``hackthenorth_b200._lib``
refuses to run without it.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libqb.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _sources():
    files = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh"))]
    files.append(os.path.join(INCLUDE, "qb.h"))
    return files


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libqb.so")


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _sources())


def nccl_dirs():
    """Headers and library of the NCCL that PyTorch loads (one libnccl.so.2 per process)."""
    import nvidia.nccl

    root = list(nvidia.nccl.__path__)[0]
    return os.path.join(root, "include"), os.path.join(root, "lib")


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    nccl_inc, nccl_lib = nccl_dirs()
    cmd = [nvcc_path(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
           "-I", INCLUDE, "-I", nccl_inc, "-o", LIB + ".tmp", os.path.join(CSRC, "qb.cu"),
           "-L", nccl_lib, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + nccl_lib]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
