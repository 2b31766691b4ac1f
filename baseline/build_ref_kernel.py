"""Build baseline/_ref/libref_noisy_gemm.so: the reference's own GPU NoisyGEMM
(miner/ampere/uwc_ampere/kernels.cu of a srivassid/useful-work-coin checkout) compiled for sm_100a
with nvcc, behind the launcher in baseline/ref_kernel_launch.cu.

    python baseline/build_ref_kernel.py [<reference checkout>]   (default: $UWC_REFERENCE)

The reference compiles this file at run time with NVRTC for the device it finds; here nvcc builds
it ahead of time with the same defines as its default configuration (-DSTAGES=3 -DBN_=128
-DMINB=2). The output is git-ignored and travels with the working tree; bench.py times it beside
this library's kernel when it exists. Nothing from the reference is copied into this repository.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "libref_noisy_gemm.so")


def build(ref: str | None = None, force: bool = False) -> str | None:
    ref = ref or os.environ.get("UWC_REFERENCE")
    src = os.path.join(ref, "miner", "ampere", "uwc_ampere", "kernels.cu") if ref else None
    if not src or not os.path.exists(src):
        return OUT if os.path.exists(OUT) else None
    launcher = os.path.join(HERE, "ref_kernel_launch.cu")
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(src),
                                                                          os.path.getmtime(launcher)):
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    cmd = [nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-DSTAGES=3", "-DBN_=128", "-DMINB=2",
           f'-DUWC_REF_KERNELS="{src}"', launcher, "-o", OUT + ".tmp"]
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, force=True))
