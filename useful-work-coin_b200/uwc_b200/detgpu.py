"""The deterministic int8 linear's fused producers and consumers on B200, with the names and
semantics of runtime/detgpu/kernels.py (quant_act, rmsnorm_quant, qkv_post, dequant_residual,
swiglu_quant) and runtime/detgpu/stages.py (linear, norm_linear), plus quant_rows_had of
miner/ampere/uwc_ampere/ops.py:172-181. Every output is bit-identical to runtime/detrt.

A linear layer `lin` is anything with `.Wq` (n x k int8, on the GPU), `.sw` (n float32) and `.bs`
(Hadamard block), e.g. detrt.qwen3.DetLinear. Its GEMM runs on this library's tcgen05 kernel with
the dequant fused into the epilogue (det.linear_f32), so no int32 matrix round-trips HBM.
"""
from __future__ import annotations

import torch

from . import det, ops
from ._lib import check, lib
from .ops import _p, _stream


def _f32(x: torch.Tensor) -> torch.Tensor:
    assert x.dtype == torch.float32 and x.is_cuda, (x.dtype, x.device)
    return x.contiguous()


def quant_act(x: torch.Tensor, bs: int) -> tuple[torch.Tensor, torch.Tensor]:
    """detrt.core.quant_act(x, bs) for float32 x (rows, k): (int8 q, float32 scale)."""
    x = _f32(x)
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty(m, dtype=torch.float32, device=x.device)
    check(lib().uwc_quant_act(_p(x), m, k, bs, _p(q), _p(s), _stream()), "quant_act")
    return q, s


def quant_rows_had(x: torch.Tensor, bs: int, q: torch.Tensor | None = None, scale: torch.Tensor | None = None):
    """x: m x k bf16 -> (int8 q in [-64, 64], float32 per-row scale), block Hadamard of size bs."""
    assert x.dtype == torch.bfloat16 and x.is_contiguous()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device) if q is None else q
    scale = torch.empty(m, dtype=torch.float32, device=x.device) if scale is None else scale
    check(lib().uwc_quant_rows_had(_p(x), m, k, bs, _p(q), _p(scale), _stream()), "quant_rows_had")
    return q, scale


def fwht_absmax(x: torch.Tensor, bs: int) -> torch.Tensor:
    """Per-row max |fwht(x, bs)| of a column shard (the row-parallel quantizer's first half)."""
    x = _f32(x)
    m, k = x.shape
    amax = torch.empty(m, dtype=torch.float32, device=x.device)
    check(lib().uwc_fwht_absmax(_p(x), m, k, bs, _p(amax), _stream()), "fwht_absmax")
    return amax


def quant_act_global(x: torch.Tensor, bs: int, amax: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quant_act of a column shard given the full row's transformed absmax (max over shards)."""
    x = _f32(x)
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty(m, dtype=torch.float32, device=x.device)
    check(lib().uwc_quant_act_global(_p(x), m, k, bs, _p(amax.contiguous()), _p(q), _p(s), _stream()),
          "quant_act_global")
    return q, s


def rmsnorm_quant(x: torch.Tensor, w: torch.Tensor, eps: float, bs: int) -> tuple[torch.Tensor, torch.Tensor]:
    """detrt.core.quant_act(detrt.core.det_rmsnorm(x, w, eps), bs) for float32 x (rows, k)."""
    x, w = _f32(x), _f32(w)
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty(m, dtype=torch.float32, device=x.device)
    check(lib().uwc_rmsnorm_quant(_p(x), _p(w), m, k, bs, float(eps), _p(q), _p(s), _stream()), "rmsnorm_quant")
    return q, s


def swiglu_quant(acc: torch.Tensor, s3: torch.Tensor, sw: torch.Tensor, bs: int) -> tuple[torch.Tensor, torch.Tensor]:
    """quant_act(det_silu(gate) * up, bs) of the gate/up GEMM's int32 output (N x 2I)."""
    acc = acc.contiguous()
    assert acc.dtype == torch.int32
    N, two_i = acc.shape
    I = two_i // 2
    q = torch.empty((N, I), dtype=torch.int8, device=acc.device)
    sc = torch.empty(N, dtype=torch.float32, device=acc.device)
    check(lib().uwc_swiglu_quant(_p(acc), _p(_f32(s3)), _p(_f32(sw)), N, I, bs, _p(q), _p(sc), _stream()),
          "swiglu_quant")
    return q, sc


def dequant_residual(acc: torch.Tensor, s: torch.Tensor, sw: torch.Tensor, x: torch.Tensor | None) -> torch.Tensor:
    """x + fmul(fmul(float(acc), s[:, None]), sw[None, :]): the residual add after o / down
    (x None: the dequantized product alone)."""
    acc = acc.contiguous()
    x = None if x is None else _f32(x)
    assert acc.dtype == torch.int32
    N, k = acc.shape
    out = torch.empty((N, k), dtype=torch.float32, device=acc.device)
    check(lib().uwc_dequant_residual(_p(acc), _p(_f32(s)), _p(_f32(sw)), _p(x), N, k, _p(out), _stream()),
          "dequant_residual")
    return out


def dequant(acc: torch.Tensor, s: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    return dequant_residual(acc, s, sw, None)


def swiglu(acc: torch.Tensor, s3: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """fp32 fmul(det_silu(gate), up) of the gate/up GEMM's int32 output (N x 2I) -> N x I."""
    acc = acc.contiguous()
    assert acc.dtype == torch.int32
    N, two_i = acc.shape
    h = torch.empty((N, two_i // 2), dtype=torch.float32, device=acc.device)
    check(lib().uwc_swiglu(_p(acc), _p(_f32(s3)), _p(_f32(sw)), N, two_i // 2, _p(h), _stream()), "swiglu")
    return h


def qkv_post(acc, s1, sw, qnw, knw, cos, sin, T: int, H: int, Hkv: int, eps: float, qknorm: bool = True):
    """Quantized q, k, v from the qkv GEMM's int32 output: (qq (N,H,128) int8, qs (N,H,1), kq, ks, vq, vs).
    qknorm False (Llama, Mistral): no per-head RMSNorm before rope."""
    acc = acc.contiguous()
    assert acc.dtype == torch.int32
    N = acc.shape[0]
    dev = acc.device
    e = lambda *shape, dt=torch.int8: torch.empty(shape, dtype=dt, device=dev)
    qq, qs = e(N, H, 128), e(N, H, 1, dt=torch.float32)
    kq, ks = e(N, Hkv, 128), e(N, Hkv, 1, dt=torch.float32)
    vq, vs = e(N, Hkv, 128), e(N, Hkv, 1, dt=torch.float32)
    qn = _f32(qnw) if qknorm else None
    kn = _f32(knw) if qknorm else None
    check(lib().uwc_qkv_post(_p(acc), _p(_f32(s1)), _p(_f32(sw)), _p(qn), _p(kn), _p(_f32(cos)), _p(_f32(sin)),
                             N, T, H, Hkv, float(eps), int(bool(qknorm)), _p(qq), _p(qs), _p(kq), _p(ks), _p(vq),
                             _p(vs), _stream()), "qkv_post")
    return qq, qs, kq, ks, vq, vs


def linear_q(lin, q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fmul(fmul(float(q @ Wq^T), s), sw): the dequantized GEMM of already-quantized rows."""
    return det.linear_f32(q, s, lin.Wq, lin.sw, static_weights=True)


def linear(lin, x: torch.Tensor) -> torch.Tensor:
    """runtime/detgpu/stages.py:85-93: quant_act, int8 GEMM, dequant (fused in the GEMM epilogue)."""
    q, s = quant_act(x, lin.bs)
    return linear_q(lin, q, s)


def norm_linear(lin, w_norm: torch.Tensor, x: torch.Tensor, eps: float) -> torch.Tensor:
    """runtime/detgpu/stages.py:96-104: linear(det_rmsnorm(x, w_norm, eps)) with the norm fused
    into the quantizer."""
    q, s = rmsnorm_quant(x, w_norm, eps, lin.bs)
    return linear_q(lin, q, s)


def linear_resid(lin, q: torch.Tensor, s: torch.Tensor, x: torch.Tensor | None) -> torch.Tensor:
    """fadd(x, deq(q @ Wq^T)): the GEMM and dequant_residual (stages.py:117-125) as one kernel, the
    residual add in the GEMM's epilogue (decode-sized rows: the weight-streaming GEMM)."""
    return ops.gemm_epi(q, lin.Wq, ops.SEPI_RESID, x_scale=s, w_scale=lin.sw, resid=x, early_w=True)


def mlp_residual(gu, down, w_norm: torch.Tensor, r1: torch.Tensor, eps: float) -> torch.Tensor:
    """The MLP half of runtime/detgpu/stages.py layer_fused (:148-153): rmsnorm_quant, gate/up GEMM,
    swiglu_quant, down GEMM, dequant_residual -- bit-identical to detrt.fast (:182-189). The SwiGLU and
    the residual add run inside the GEMMs' epilogues (quant_act of the SwiGLU row is swiglu_quant's
    second half), so no int32 product goes through HBM."""
    q3, s3 = rmsnorm_quant(r1, w_norm, eps, gu.bs)
    if gu.Wq.shape[0] % 8 == 0:
        h = ops.gemm_epi(q3, gu.Wq, ops.SEPI_SWIGLU, x_scale=s3, w_scale=gu.sw, early_w=True)
        q4, s4 = quant_act(h, down.bs)
    else:
        q4, s4 = swiglu_quant(det.int_gemm(q3, gu.Wq), s3, gu.sw, down.bs)
    return linear_resid(down, q4, s4, r1)


TC_MIN_ROWS = 128        # query rows per sequence from which attention runs its GEMMs on tcgen05
TC_MAX_KEYS = 12800      # the tensor-core softmax keeps 4 query rows' scores in shared memory
TC_MAX_WORKSPACE = 24 << 30   # larger calls (long prompts times many heads) run the SIMT kernel
_TC_WS: dict = {}         # device -> workspace of the tensor-core attention (grown on demand)


def use_tensor_cores(B: int, Tq: int, start: int, H: int, Hkv: int, path: str = "auto") -> bool:
    """Whether attention of Tq query rows per sequence runs on the tensor-core path: forced by
    path "tc" / "simt", else from TC_MIN_ROWS rows while the keys fit the softmax pass's shared
    memory and the workspace (int32 scores, P limbs) stays within TC_MAX_WORKSPACE bytes."""
    if path in ("tc", "simt"):
        return path == "tc"
    if path != "auto":
        raise ValueError(f"attention path {path!r}")
    if Tq < TC_MIN_ROWS or start + Tq > TC_MAX_KEYS:
        return False
    return int(lib().uwc_attention_tc_workspace_bytes(B, Tq, start, H, Hkv)) <= TC_MAX_WORKSPACE


def _tc_workspace(device, nbytes: int) -> torch.Tensor:
    ws = _TC_WS.get(str(device))
    if ws is None or ws.numel() < nbytes:
        _TC_WS[str(device)] = ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
    return ws


def _attn(qq, qs, kc, ks, vc, vs, B, Tq, start, H, Hkv, strides, inv_sqrt_hd, path: str = "auto") -> torch.Tensor:
    """path: "simt" (one CTA per block of query rows, dp4a dots), "tc" (Q K^T and P V as batched
    tcgen05 GEMMs), or "auto" (tc from TC_MIN_ROWS query rows per sequence). Same bits either way."""
    assert qq.dtype == torch.int8 and qq.shape[-1] == 128 and qq.is_contiguous(), (qq.dtype, qq.shape)
    out = torch.empty((B * Tq, H * 128), dtype=torch.float32, device=qq.device)
    if use_tensor_cores(B, Tq, start, H, Hkv, path):
        need = int(lib().uwc_attention_tc_workspace_bytes(B, Tq, start, H, Hkv))
        ws = _tc_workspace(qq.device, need)
        check(lib().uwc_attention_tc(_p(qq), _p(_f32(qs)), _p(kc), _p(ks), _p(vc), _p(vs), B, Tq, start, H, Hkv,
                                     *strides, float(inv_sqrt_hd), _p(out), _p(ws), ws.numel(), _stream()),
              "attention_tc")
        return out
    check(lib().uwc_attention(_p(qq), _p(_f32(qs)), _p(kc), _p(ks), _p(vc), _p(vs), B, Tq, start, H, Hkv, *strides,
                              float(inv_sqrt_hd), _p(out), _stream()), "attention")
    return out


def attention(qq, qs, kq, ks, vq, vs, B: int, T: int, H: int, Hkv: int, inv_sqrt_hd_f32: float,
              path: str = "auto") -> torch.Tensor:
    """runtime/detgpu/kernels.py attention: detrt's attention of B sequences of T tokens from
    quantized q, k, v -- qq (N, H, 128), kq and vq (N, Hkv, 128) int8, qs (N, H, 1), ks and vs
    (N, Hkv, 1) float32, N = B * T. Returns o as (N, H * 128) float32."""
    i8 = lambda z: z.to(torch.int8).contiguous()
    kq, vq = i8(kq), i8(vq)
    ks, vs = _f32(ks), _f32(vs)
    strides = (T * Hkv * 128, Hkv * 128, 128, T * Hkv, Hkv, 1)
    return _attn(i8(qq), qs, kq, ks, vq, vs, B, T, 0, H, Hkv, strides, inv_sqrt_hd_f32, path)


def attention_cache(qq, qs, cache: dict, B: int, Tq: int, start: int, H: int, Hkv: int,
                    inv_sqrt_hd_f32: float, path: str = "auto") -> torch.Tensor:
    """Attention of Tq new tokens per sequence (positions start .. start + Tq - 1) over a KV cache
    laid out as runtime/detrt/qwen3.py new_cache: k, v (B, Hkv, maxlen, 128) int8, sk, sv
    (B, Hkv, maxlen, 1) float32, already holding keys 0 .. start + Tq - 1 (qwen3.py:254-283)."""
    k, v, sk, sv = cache["k"], cache["v"], cache["sk"], cache["sv"]
    assert k.is_contiguous() and v.is_contiguous() and sk.is_contiguous() and sv.is_contiguous()
    maxlen = k.shape[2]
    assert start + Tq <= maxlen
    strides = (Hkv * maxlen * 128, 128, maxlen * 128, Hkv * maxlen, 1, maxlen)
    return _attn(qq.contiguous(), qs, k, sk, v, sv, B, Tq, start, H, Hkv, strides, inv_sqrt_hd_f32, path)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """detrt.core.det_rmsnorm(x, w, eps) for float32 rows."""
    x, w = _f32(x), _f32(w)
    m, k = x.shape
    out = torch.empty_like(x)
    check(lib().uwc_rmsnorm(_p(x), _p(w), m, k, float(eps), _p(out), _stream()), "rmsnorm")
    return out


def logprobs(logits: torch.Tensor, want_lp: bool = True):
    """DetQwen3.logprobs rows (runtime/detrt/qwen3.py:302-312) and the greedy tokens (the first
    index of each row's maximal log-probability): (lp or None, tokens int64)."""
    lg = _f32(logits)
    m, V = lg.shape
    lp = torch.empty_like(lg) if want_lp else None
    tok = torch.empty(m, dtype=torch.int64, device=lg.device)
    check(lib().uwc_logprobs(_p(lg), m, V, _p(lp), _p(tok), _stream()), "logprobs")
    return lp, tok


def qkv_post_at(acc, s1, sw, qnw, knw, cos_table, sin_table, pos: torch.Tensor, T: int, H: int, Hkv: int, eps: float,
                qknorm: bool = True):
    """qkv_post with the rope rows at the device-side position pos (int32, one element) + r % T."""
    acc = acc.contiguous()
    assert acc.dtype == torch.int32 and pos.dtype == torch.int32
    N = acc.shape[0]
    dev = acc.device
    e = lambda *shape, dt=torch.int8: torch.empty(shape, dtype=dt, device=dev)
    qq, qs = e(N, H, 128), e(N, H, 1, dt=torch.float32)
    kq, ks = e(N, Hkv, 128), e(N, Hkv, 1, dt=torch.float32)
    vq, vs = e(N, Hkv, 128), e(N, Hkv, 1, dt=torch.float32)
    qn = _f32(qnw) if qknorm else None
    kn = _f32(knw) if qknorm else None
    check(lib().uwc_qkv_post_at(_p(acc), _p(_f32(s1)), _p(_f32(sw)), _p(qn), _p(kn), _p(_f32(cos_table)),
                                _p(_f32(sin_table)), _p(pos), N, T, H, Hkv, float(eps), int(bool(qknorm)), _p(qq),
                                _p(qs), _p(kq), _p(ks), _p(vq), _p(vs), _stream()), "qkv_post_at")
    return qq, qs, kq, ks, vq, vs


def qkv_post_kv(acc, s1, sw, qnw, knw, cos_table, sin_table, pos: torch.Tensor, T: int, H: int, Hkv: int, eps: float,
                cache: dict, qknorm: bool = True):
    """qkv_post_at with the keys / values stored straight into `cache` at pos (+ r % T): the
    qkv_post_at + kv_append pair of a decode step in one kernel. Returns (qq, qs)."""
    acc = acc.contiguous()
    assert acc.dtype == torch.int32 and pos.dtype == torch.int32
    N = acc.shape[0]
    qq = torch.empty((N, H, 128), dtype=torch.int8, device=acc.device)
    qs = torch.empty((N, H, 1), dtype=torch.float32, device=acc.device)
    k, v, sk, sv = cache["k"], cache["v"], cache["sk"], cache["sv"]
    assert k.shape[1] == Hkv and k.is_contiguous() and v.is_contiguous() and sk.is_contiguous() and sv.is_contiguous()
    qn = _f32(qnw) if qknorm else None
    kn = _f32(knw) if qknorm else None
    check(lib().uwc_qkv_post_kv(_p(acc), _p(_f32(s1)), _p(_f32(sw)), _p(qn), _p(kn), _p(_f32(cos_table)),
                                _p(_f32(sin_table)), _p(pos), N, T, H, Hkv, float(eps), int(bool(qknorm)), _p(qq),
                                _p(qs), _p(k), _p(sk), _p(v), _p(sv), k.shape[2], _stream()), "qkv_post_kv")
    return qq, qs


def kv_append(kq, ks, vq, vs, cache: dict, B: int, T: int, pos: torch.Tensor) -> None:
    """Write the new tokens' keys / values into the cache at the device-side position pos."""
    k, v, sk, sv = cache["k"], cache["v"], cache["sk"], cache["sv"]
    Hkv, maxlen = k.shape[1], k.shape[2]
    check(lib().uwc_kv_append(_p(kq.contiguous()), _p(_f32(ks)), _p(vq.contiguous()), _p(_f32(vs)), B, T, Hkv, maxlen,
                              _p(pos), _p(k), _p(sk), _p(v), _p(sv), _stream()), "kv_append")


def attention_cache_at(qq, qs, cache: dict, B: int, Tq: int, pos: torch.Tensor, max_start: int, H: int, Hkv: int,
                       inv_sqrt_hd_f32: float) -> torch.Tensor:
    """attention_cache with the start position read from device memory (pos <= max_start)."""
    k, v, sk, sv = cache["k"], cache["v"], cache["sk"], cache["sv"]
    maxlen = k.shape[2]
    assert max_start + Tq <= maxlen and pos.dtype == torch.int32
    qq = qq.contiguous()
    out = torch.empty((B * Tq, H * 128), dtype=torch.float32, device=qq.device)
    strides = (Hkv * maxlen * 128, 128, maxlen * 128, Hkv * maxlen, 1, maxlen)
    check(lib().uwc_attention_at(_p(qq), _p(_f32(qs)), _p(k), _p(sk), _p(v), _p(sv), B, Tq, _p(pos), max_start, H,
                                 Hkv, *strides, float(inv_sqrt_hd_f32), _p(out), _stream()), "attention_at")
    return out
