"""Build ``libfrattn.so`` in-tree with nvcc for sm_100a.

``python -m fused_rope_attn_b200.build`` (or ``__graft_entry__.build()``).
The kernels of each supported head dimension are compiled from
``csrc/frattn_inst.cu`` into their own object (``-DFRATTN_D=<D>``), in
parallel, and linked with the host code of ``csrc/frattn.cu`` into one shared
library. The CUDA runtime is linked statically so the library loads on
machines without a GPU (the C-ABI symbol test) and needs only the driver at
run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
HOST_SRC = os.path.join(CSRC, "frattn.cu")
INST_SRC = os.path.join(CSRC, "frattn_inst.cu")
WINDOW_SRC = os.path.join(CSRC, "frattn_window.cu")
QKV_SRC = os.path.join(CSRC, "frattn_qkv.cu")
BWD_SRC = os.path.join(CSRC, "frattn_bwd.cu")
FP8_SRC = os.path.join(CSRC, "frattn_fp8.cu")
DEPS = [HOST_SRC, INST_SRC, WINDOW_SRC, QKV_SRC, BWD_SRC, FP8_SRC, os.path.join(CSRC, "frattn_kernel.cuh"), os.path.join(CSRC, "frattn_ptx.cuh"),
        os.path.join(ROOT, "include", "frattn.h")]
OUT = os.path.join(HERE, "libfrattn.so")
OBJ_DIR = os.path.join(HERE, "_build")

HEAD_DIMS = tuple(range(32, 129, 8))  # must match FRATTN_HEAD_DIMS in csrc/frattn.cu

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC",
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


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(OBJ_DIR, exist_ok=True)
    extra = ["-Xptxas=-v"] if verbose else []
    jobs = jobs or max(1, os.cpu_count() or 1)
    cmds, objs = [], []
    for d in HEAD_DIMS:
        obj = os.path.join(OBJ_DIR, f"frattn_d{d}.o")
        cmds.append([nvcc(), *NVCC_FLAGS, *extra, f"-DFRATTN_D={d}", "-c", "-o", obj, INST_SRC])
        objs.append(obj)
    win_obj = os.path.join(OBJ_DIR, "frattn_window.o")
    cmds.append([nvcc(), *NVCC_FLAGS, *extra, "-c", "-o", win_obj, WINDOW_SRC])
    objs.append(win_obj)
    fp8_obj = os.path.join(OBJ_DIR, "frattn_fp8.o")
    cmds.append([nvcc(), *NVCC_FLAGS, *extra, "-c", "-o", fp8_obj, FP8_SRC])
    objs.append(fp8_obj)
    bwd_obj = os.path.join(OBJ_DIR, "frattn_bwd.o")
    cmds.append([nvcc(), *NVCC_FLAGS, *extra, "-c", "-o", bwd_obj, BWD_SRC])
    objs.append(bwd_obj)
    qkv_obj = os.path.join(OBJ_DIR, "frattn_qkv.o")
    cmds.append([nvcc(), *NVCC_FLAGS, *extra, "-c", "-o", qkv_obj, QKV_SRC])
    objs.append(qkv_obj)
    host_obj = os.path.join(OBJ_DIR, "frattn_host.o")
    cmds.append([nvcc(), *NVCC_FLAGS, *extra, "-c", "-o", host_obj, HOST_SRC])
    objs.append(host_obj)
    # the slowest objects first
    with ThreadPoolExecutor(max_workers=jobs) as pool:
        for f in [pool.submit(_run, c, verbose) for c in cmds]:
            f.result()
    tmp = OUT + ".tmp"
    _run([nvcc(), "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a", "-o", tmp,
          *objs], verbose)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
