"""Build libuwcb200.so (the C-ABI library) for sm_100a with nvcc, in-tree.

    python useful-work-coin_b200/build.py [--force] [--verbose]

Output: useful-work-coin_b200/uwc_b200/libuwcb200.so, linked against the static CUDA runtime so
it loads on a machine without a GPU driver (the symbol-export test runs on CPU-only hosts).
Nothing is compiled at import time: the product path refuses to run without this library.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "uwc_b200", "libuwcb200.so")
SOURCES = ["host.cu", "prep.cu", "gemm_sm100.cu", "mined.cu", "peak.cu", "stream_gemm.cu", "tp.cu", "detq.cu", "attn.cu", "sha.cu"]
HEADERS = ["uwc_device.cuh", "uwc_host.h", "det_math.cuh", "uwc_tp.cuh"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-cudart", "static"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _inputs():
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(ROOT, "include", "uwc_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc(), *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = OUT + ".tmp"
    subprocess.check_call([nvcc(), "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a",
                           *objs, "-o", tmp])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    sys.exit(0)
