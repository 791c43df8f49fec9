"""Builds ``libkappa_w8.so`` in-tree with nvcc for sm_100a.

    python -m kappa_b200.build [--force] [-v]

The library is one translation unit (``csrc/kappa_w8.cu``) compiled with
``-gencode arch=compute_100a,code=sm_100a``; nvcc cross-compiles without a
GPU.  The output lands next to this file, where ``kappa_b200._lib`` loads it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc", "kappa_w8.cu")
OUT = os.path.join(HERE, "libkappa_w8.so")

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    d = os.path.join(HERE, "csrc")
    return sorted(os.path.join(d, f) for f in os.listdir(d) if f.endswith((".cu", ".cuh")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = sources() + [os.path.join(os.path.dirname(HERE), "include", "kappa_w8.h")]
    return all(os.path.getmtime(p) <= t for p in deps if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library unless it is newer than its sources; return its path."""
    if not force and up_to_date():
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", tmp, SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
