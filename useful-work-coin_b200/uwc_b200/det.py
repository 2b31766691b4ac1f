"""The deterministic int8 linear of runtime/detrt on B200 (runtime/detrt/qwen3.py:71-126).

`int_gemm(q, Wq)` is DetLinear.int_gemm's exact q @ Wq^T (int32), and `linear_f32` fuses the
dequant y = fmul(fmul(float(acc), s_x), s_w) (qwen3.py:125, detgpu/kernels.py:35) into the GEMM
epilogue, so the int32 matrix never round-trips HBM. Both run on the tcgen05 kernel; integer
accumulation is exact, so results are bit-identical to the CPU float64 path for any m.
"""
from __future__ import annotations

import torch

from . import ops


def int_gemm(q: torch.Tensor, Wq: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Exact q @ Wq^T for int8 q (m x k) and Wq (n x k), int32 result (DetLinear.int_gemm)."""
    m, n = q.shape[0], Wq.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.int32, device=q.device)
    ops.gemm(q.contiguous(), Wq.contiguous(), out=out, out_mode=ops.OUT_I32)
    return out


def linear_f32(q: torch.Tensor, s_x: torch.Tensor, Wq: torch.Tensor, s_w: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """fmul(fmul(float32(q @ Wq^T), s_x[:, None]), s_w[None, :]) in one kernel (fp32 out)."""
    m, n = q.shape[0], Wq.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=q.device)
    ops.gemm(q.contiguous(), Wq.contiguous(), a_scale=s_x.contiguous().float(), b_scale=s_w.contiguous().float(),
             out=out, out_mode=ops.OUT_F32)
    return out


def patch_detlinear(DetLinear) -> None:
    """Route DetLinear.int_gemm (qwen3.py:106-119) through this library for CUDA devices, the way
    runtime/agent/mining.py:49-65 monkey-patches it; the CPU path stays the reference's."""
    orig = DetLinear.int_gemm

    def int_gemm_b200(self, q):
        if self.device.type != "cuda":
            return orig(self, q)
        return int_gemm(q, self.Wq)

    DetLinear.int_gemm = int_gemm_b200
