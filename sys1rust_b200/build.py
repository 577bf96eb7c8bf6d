"""Build ``libs1c.so`` in-tree with nvcc for sm_100a.

``python -m sys1rust_b200.build`` (or ``__graft_entry__.build()``) compiles
``sys1rust_b200/csrc/s1c.cu`` into ``sys1rust_b200/libs1c.so``. The library links only the CUDA
runtime; the driver's tensor-map encoder is looked up at run time.
"""
from __future__ import annotations

import fcntl
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libs1c.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list:
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(ROOT, "include", "s1c.h"), os.path.abspath(__file__)]
    return all(os.path.getmtime(p) <= t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library unless it is newer than every source. Safe to call from several
    processes at once (e.g. every rank of a torchrun job): one compiles under a file lock while the
    others wait and then find the library up to date."""
    if not force and up_to_date():
        return LIB
    with open(LIB + ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and up_to_date():
            return LIB
        return _compile(verbose)


def _compile(verbose: bool) -> str:
    tmp = f"{LIB}.{os.getpid()}.tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-shared", "-o", tmp, os.path.join(CSRC, "s1c.cu"), "-lcudart"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
