"""The deterministic int8 linear of runtime/detrt on B200 (runtime/detrt/qwen3.py:71-126).

`int_gemm(q, Wq)` is DetLinear.int_gemm's exact q @ Wq^T (int32), and `linear_f32` fuses the
dequant y = fmul(fmul(float(acc), s_x), s_w) (qwen3.py:125, detgpu/kernels.py:35) into the GEMM
epilogue, so the int32 matrix never round-trips HBM. Both run on the tcgen05 kernel; integer
accumulation is exact, so results are bit-identical to the CPU float64 path for any m.
"""
from __future__ import annotations

import torch

from . import ops


def int_gemm(q: torch.Tensor, Wq: torch.Tensor, out: torch.Tensor | None = None,
             static_weights: bool = False) -> torch.Tensor:
    """Exact q @ Wq^T for int8 q (m x k) and Wq (n x k), int32 result (DetLinear.int_gemm).
    static_weights: Wq is a model weight, not produced by the kernel just before this call, so a
    decode-sized call may start streaming it early (ops.gemm_stream's early_w)."""
    m, n = q.shape[0], Wq.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.int32, device=q.device)
    if static_weights and m <= ops.STREAM_MAX_M:
        return ops.gemm_stream(q.contiguous(), Wq.contiguous(), ops.SEPI_I32, out=out, early_w=True)
    ops.gemm(q.contiguous(), Wq.contiguous(), out=out, out_mode=ops.OUT_I32)
    return out


def linear_f32(q: torch.Tensor, s_x: torch.Tensor, Wq: torch.Tensor, s_w: torch.Tensor,
               out: torch.Tensor | None = None, static_weights: bool = False) -> torch.Tensor:
    """fmul(fmul(float32(q @ Wq^T), s_x[:, None]), s_w[None, :]) in one kernel (fp32 out)."""
    m, n = q.shape[0], Wq.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=q.device)
    if static_weights and m <= ops.STREAM_MAX_M:
        return ops.gemm_stream(q.contiguous(), Wq.contiguous(), ops.SEPI_F32, x_scale=s_x, w_scale=s_w, out=out,
                               early_w=True)
    ops.gemm(q.contiguous(), Wq.contiguous(), a_scale=s_x.contiguous().float(), b_scale=s_w.contiguous().float(),
             out=out, out_mode=ops.OUT_F32)
    return out


def patch_detlinear(DetLinear) -> None:
    """Route DetLinear.int_gemm (runtime/detrt/qwen3.py:106-119) through this library on CUDA devices,
    the way runtime/agent/mining.py:49-65 patches it for mining: a layer that mines with one of this
    library's MinedWeights (lin.mine and lin.mw) runs the hashed forward on its rows padded to a
    multiple of 64 (int32 out, unit scales); any other CUDA layer gets the exact int32 q @ Wq^T of
    the tcgen05 GEMM. CPU layers keep the reference's own float64 path. The original method stays
    reachable as DetLinear._orig_int_gemm; patching twice is a no-op."""
    if getattr(DetLinear, "_uwc_b200_patched", False):
        return
    orig = DetLinear.int_gemm

    def int_gemm_b200(self, q):
        if self.device.type != "cuda":
            return orig(self, q)
        mw = getattr(self, "mw", None)
        if getattr(self, "mine", False) and isinstance(mw, ops.MinedWeight):
            m = q.shape[0]
            mp = -(-m // 64) * 64
            qp = torch.nn.functional.pad(q, (0, 0, 0, mp - m)) if mp != m else q
            ones = torch.ones(mp, dtype=torch.float32, device=q.device)
            return mw.forward(qp.contiguous(), ones, out_mode=ops.OUT_I32)[:m]
        return int_gemm(q, self.Wq)

    DetLinear._orig_int_gemm = orig
    DetLinear.int_gemm = int_gemm_b200
    DetLinear._uwc_b200_patched = True
