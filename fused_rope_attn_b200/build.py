"""Build ``libfrattn.so`` in-tree with nvcc for sm_100a.

``python -m fused_rope_attn_b200.build`` (or ``__graft_entry__.build()``).
The CUDA runtime is linked statically so the library loads on machines
without a GPU (the C-ABI symbol test) and needs only the driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "frattn.cu")
DEPS = [SRC, os.path.join(HERE, "csrc", "frattn_ptx.cuh"), os.path.join(ROOT, "include", "frattn.h")]
OUT = os.path.join(HERE, "libfrattn.so")

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
    "-I", os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(d) <= t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", tmp, SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
