"""uwc_b200: the cuPOW NoisyGEMM hot path of useful-work-coin, rebuilt for B200 (sm_100a).

Modules:
  ops   drop-in for miner/ampere/uwc_ampere/ops.py (launchers, MinedWeight, GraphedForward)
  det   the deterministic int8 linear of runtime/detrt (DetLinear.int_gemm and its fp32 dequant)
  glue  host-side target/bound helpers of miner/ampere/uwc_ampere/pearl_glue.py
The kernels live in libuwcb200.so (C ABI: include/uwc_b200.h), built by ../build.py.
"""
__all__ = ["ops", "det", "glue"]
