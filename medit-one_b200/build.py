"""Build libone_b200.so (the sm_100a engine) in-tree with nvcc.

    python medit-one_b200/build.py [--force]

The library is a plain C-ABI shared object (include/one_b200.h): no torch headers,
compiled for sm_100a only. It lands in medit-one_b200/one/libone_b200.so, where the
`one` package loads it.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "one", "libone_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
         "-Xcompiler", "-fPIC", "-shared", "-diag-suppress=177"]


def _sources():
    files = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))
    files.append(os.path.join(os.path.dirname(HERE), "include", "one_b200.h"))
    return files


def _digest():
    h = hashlib.sha256()
    for f in _sources():
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = True) -> str:
    stamp = OUT + ".sha256"
    dig = _digest()
    if not force and os.path.exists(OUT) and os.path.exists(stamp) and open(stamp).read().strip() == dig:
        return OUT
    cmd = [NVCC, *FLAGS, "-o", OUT, os.path.join(CSRC, "engine.cu"), os.path.join(CSRC, "linear_moe_noalloc.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    with open(stamp, "w") as fh:
        fh.write(dig)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv)
