"""Builds libforgegpu.so (the C-ABI engine) for sm_100a with nvcc, in-tree.

Usage: python forge-db_b200/build.py [--jobs N] [--force]
The library lands in forge-db_b200/forgegpu/libforgegpu.so, next to the
ctypes binding that loads it.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "forgegpu", "libforgegpu.so")
SOURCES = ["capi.cu", "engine.cu", "distances.cu", "kmeans.cu", "pq.cu", "ivfpq_kernels.cu",
           "bf_kernels.cu", "gemm_topk.cu", "ivf_tc.cu", "coarse_tc.cu", "mutate.cu", "persist.cu"]
HEADERS = ["fdb_device.cuh", "fdb_internal.h", "fdb_kernels.h", "tc_ptx.cuh"]

NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_home() -> tuple[str, str]:
    """(include dir, lib dir) of the NCCL to build against.

    PyTorch ships its own libnccl.so.2 (the nvidia-nccl wheel).  A process
    that loads a second libnccl.so.2 first (the system one) breaks torch's
    later import with missing symbols, so link the wheel's copy when it is
    there: both libraries then share one NCCL."""
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is not None and spec.submodule_search_locations:
        for base in spec.submodule_search_locations:
            inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
            if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(
                    os.path.join(lib, "libnccl.so.2")):
                return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


NCCL_INC, NCCL_LIB = _nccl_home()
# -fmad=false: no compiler contraction of a*b+c; every fused multiply-add in
# the kernels is an explicit __fmaf_rn, so summation orders match the
# reference's AVX2 arithmetic bit for bit.
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC,-O2",
                "-ccbin", "g++", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
                "-I", NCCL_INC]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(OBJ, src.replace(".cu", ".o"))
    deps = [os.path.join(CSRC, src)] + [os.path.join(CSRC, h) for h in HEADERS] + [
        os.path.join(ROOT, "include", "forgegpu.h")]
    if force or _newer(obj, deps):
        cmd = [NVCC] + FLAGS + ["-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(jobs: int = 8, force: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or _newer(OUT, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", OUT + ".tmp"] + objs + [
            "-cudart", "static", "-L", NCCL_LIB, "-l:libnccl.so.2", "-Xlinker",
            "-rpath," + NCCL_LIB]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        shutil.move(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.force))
    sys.exit(0)
