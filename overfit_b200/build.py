"""Builds libovf_cuda.so in-tree for sm_100a (B200).

The library is plain CUDA C++ with a C ABI (include/ovf.h); no torch types
cross the boundary, so it is compiled with nvcc directly rather than as a
torch extension.  Output: overfit_b200/libovf_cuda.so.
"""
from __future__ import annotations

import fcntl
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libovf_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  [os.path.join(ROOT, "include", "ovf.h")])


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compiles the library unless it is newer than every source.  Several
    processes may call this at once (one per rank under torchrun): a file
    lock serialises them, and the ones that waited find the library built."""
    if not force and up_to_date():
        return LIB
    with open(os.path.join(HERE, ".build.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and up_to_date():
                return LIB
            tmp = f"{LIB}.{os.getpid()}.tmp"
            cmd = [nvcc(), *ARCH, *FLAGS, *(extra or []), "-I", os.path.join(ROOT, "include"),
                   "-o", tmp, os.path.join(CSRC, "ovf_lib.cu")]
            if verbose:
                print(" ".join(cmd))
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError("nvcc failed building libovf_cuda.so")
            if verbose and (r.stdout or r.stderr):
                print(r.stdout + r.stderr)
            os.replace(tmp, LIB)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
