"""CPU oracle for the deterministic int8 linear's producers and consumers -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may import this module.

A numpy restatement of runtime/detrt's emulated-fp32 primitives (paths inside
srivassid/useful-work-coin) and of the fused detgpu row kernels built from them:

  fadd / fsub / fmul / fdiv / fsqrt (one rounding per op)   runtime/detrt/core.py:53-70
  pow2_f32, pow2_f64                                         runtime/detrt/core.py:74-82
  exact_rowsum (int64 fixed point, row-max scale)            runtime/detrt/core.py:85-108
  det_exp (degree-7 2^f polynomial), det_silu                runtime/detrt/core.py:103-127,146-148
  det_rmsnorm                                                runtime/detrt/core.py:151-159
  quant_sym, fwht, quant_act                                 runtime/detrt/core.py:162-196
  deq = fmul(fmul(float(acc), s), sw)                        runtime/detgpu/kernels.py:35
  rmsnorm_quant (norm fused into the quantizer)              runtime/detgpu/kernels.py:117-191
  qkv_post (dequant, q/k head RMSNorm, rope, quant_sym 127)  runtime/detgpu/kernels.py:303-344,
                                                             runtime/detrt/fast.py:108-120
  dequant_residual (x + deq(acc))                            runtime/detgpu/kernels.py:346-354
  swiglu_quant (quant_act(silu(gate) * up))                  runtime/detgpu/kernels.py:356-396
  attention (exact Q K^T, det_exp softmax, 14-bit P, exact PV) runtime/detrt/qwen3.py:253-283
  det_log, logprobs                                          runtime/detrt/core.py:130-143,
                                                             runtime/detrt/qwen3.py:302-312
  int_gemm, quantize_linear, layer_forward                   runtime/detrt/qwen3.py:71-126,239-297

numpy float32 arithmetic on x86-64 is IEEE single precision with one rounding per operation,
which is exactly detrt's float64-then-round emulation for + - * / sqrt; the helpers below still
spell the float64 round trip out. Pinned by tests/test_det_oracle.py and tests/test_model_oracle.py
against vectors that tests/golden/make_golden_det.py and make_golden_model.py produced with detrt
itself (the layer composition reproduces detrt's whole prefill forward of a tiny Qwen3).
"""
from __future__ import annotations

import math

import numpy as np

F32, F64 = np.float32, np.float64

# detrt.core._EXP2 / _LOG2E (core.py:100-102): the project's own exp polynomial
EXP2 = [1.0, 0.6931471824645996, 0.2402263879776001, 0.055505119264125824, 0.00961404386907816,
        0.001342222560197115, 0.0001435537706129253, 2.1489791834028438e-05]
LOG2E = 1.4426950408889634


def c32(v: float) -> np.float32:
    return F32(F64(v))


def fadd(a, b):
    return (np.asarray(a, F32).astype(F64) + np.asarray(b, F32).astype(F64)).astype(F32)


def fsub(a, b):
    return (np.asarray(a, F32).astype(F64) - np.asarray(b, F32).astype(F64)).astype(F32)


def fmul(a, b):
    return (np.asarray(a, F32).astype(F64) * np.asarray(b, F32).astype(F64)).astype(F32)


def fdiv(a, b):
    return (np.asarray(a, F32).astype(F64) / np.asarray(b, F32).astype(F64)).astype(F32)


def fsqrt(a):
    return np.sqrt(np.asarray(a, F32).astype(F64)).astype(F32)


def pow2_f32(n):
    return ((np.asarray(n).astype(np.int32) + 127) << 23).astype(np.int32).view(F32)


def pow2_f64(n):
    return ((np.asarray(n).astype(np.int64) + 1023) << 52).astype(np.int64).view(F64)


def exact_rowsum(x: np.ndarray, max_terms: int) -> np.ndarray:
    """Order-independent row sum: each term rounded once to int64 at 2^shift (core.py:85-108)."""
    x = np.asarray(x, F32)
    L = max(1, math.ceil(math.log2(max_terms)))
    amax = np.abs(x).max(axis=-1, keepdims=True)
    _, e = np.frexp(amax)
    shift = np.clip((62 - L) - e.astype(np.int64), -1000, 1000)
    q = np.rint(x.astype(F64) * pow2_f64(shift)).astype(np.int64)
    s = q.sum(axis=-1, keepdims=True)
    return (s.astype(F64) * pow2_f64(-shift)).astype(F32)[..., 0]


def det_exp(z: np.ndarray) -> np.ndarray:
    z = np.asarray(z, F32)
    t = fmul(z, c32(LOG2E))
    under = t < c32(-126.0)
    over = t >= c32(128.0)
    t = np.where(under | over | np.isnan(t), F32(0), t).astype(F32)
    n = np.floor(t).astype(F32)
    f = fsub(t, n)
    p = np.full_like(f, c32(EXP2[7]))
    for cf in reversed(EXP2[:7]):
        p = fadd(fmul(p, f), c32(cf))
    r = fmul(p, pow2_f32(n))
    r = np.where(under, F32(0), r)
    r = np.where(over, F32(np.inf), r)
    return np.where(np.isnan(z), z, r).astype(F32)


def det_silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, F32)
    return fdiv(x, fadd(c32(1.0), det_exp(-x)))


def det_rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, F32)
    d = x.shape[-1]
    ss = exact_rowsum(fmul(x, x), d)
    mean = fmul(ss, c32(1.0 / d))
    r = fdiv(c32(1.0), fsqrt(fadd(mean, c32(eps))))
    return fmul(fmul(x, r[..., None]), np.asarray(w, F32))


def quant_sym(x: np.ndarray, qmax: int):
    x = np.asarray(x, F32)
    amax = np.abs(x).max(axis=-1, keepdims=True)
    s = fdiv(np.maximum(amax, c32(1e-8)), c32(float(qmax)))
    q = np.clip(np.rint(fdiv(x, s)), -qmax, qmax)
    return q, s


def fwht(x: np.ndarray, bs: int) -> np.ndarray:
    """Unnormalized block Walsh-Hadamard transform, stages h = 1, 2, 4, ...: (a, b) -> (a+b, a-b)."""
    v = np.asarray(x, F32)
    if bs <= 1:
        return v.copy()
    shp = v.shape
    k = shp[-1]
    v = v.reshape(-1, k)
    h = 1
    while h < bs:
        v = v.reshape(v.shape[0], k // (2 * h), 2, h)
        a, b = v[:, :, 0, :], v[:, :, 1, :]
        v = np.stack([fadd(a, b), fsub(a, b)], axis=2).reshape(-1, k)
        h *= 2
    return v.reshape(shp)


def quant_act(x: np.ndarray, bs: int, qmax: int = 64):
    """(int8 q, float32 scale) with the 1/sqrt(bs) normalization folded into the scale."""
    y = fwht(x, bs)
    q, s = quant_sym(y, qmax)
    if bs > 1:
        s = fmul(s, fdiv(c32(1.0), fsqrt(c32(float(bs)))))
    return q.astype(np.int8), s[..., 0]


def quant_act_global(x: np.ndarray, bs: int, amax: np.ndarray, qmax: int = 64):
    """quant_act of a column shard whose row absmax (of the transformed row) is `amax`, the max
    over all shards: the row-parallel tensor-parallel form. Same q and scale as the full row."""
    y = fwht(x, bs)
    s = fdiv(np.maximum(np.asarray(amax, F32)[:, None], c32(1e-8)), c32(float(qmax)))
    q = np.clip(np.rint(fdiv(y, s)), -qmax, qmax)
    if bs > 1:
        s = fmul(s, fdiv(c32(1.0), fsqrt(c32(float(bs)))))
    return q.astype(np.int8), s[..., 0]


def fwht_absmax(x: np.ndarray, bs: int) -> np.ndarray:
    return np.abs(fwht(x, bs)).max(axis=-1)


def deq(acc: np.ndarray, s: np.ndarray, sw: np.ndarray) -> np.ndarray:
    return fmul(fmul(np.asarray(acc, np.int32).astype(F32), np.asarray(s, F32)[:, None]), np.asarray(sw, F32)[None, :])


def rmsnorm_quant(x: np.ndarray, w: np.ndarray, eps: float, bs: int):
    return quant_act(det_rmsnorm(x, w, eps), bs)


def dequant_residual(acc: np.ndarray, s: np.ndarray, sw: np.ndarray, x: np.ndarray) -> np.ndarray:
    return fadd(np.asarray(x, F32), deq(acc, s, sw))


def swiglu_quant(acc: np.ndarray, s3: np.ndarray, sw: np.ndarray, bs: int):
    I = acc.shape[1] // 2
    gu = deq(acc, s3, sw)
    return quant_act(fmul(det_silu(gu[:, :I]), gu[:, I:]), bs)


def qkv_post(acc, s1, sw, qnw, knw, cos, sin, T: int, H: int, Hkv: int, eps: float, qknorm: bool = True):
    """(qq (N,H,128) int8, qs (N,H,1) f32, kq, ks, vq, vs) from the qkv GEMM's int32 output.
    Row r of acc is token position r % T; cos / sin are (T or more, 128) float32 tables."""
    hd = 128
    N = acc.shape[0]
    qkv = deq(acc, s1, sw)
    q = qkv[:, :H * hd].reshape(N, H, hd)
    k = qkv[:, H * hd:(H + Hkv) * hd].reshape(N, Hkv, hd)
    v = qkv[:, (H + Hkv) * hd:].reshape(N, Hkv, hd)
    if qknorm:
        q = det_rmsnorm(q, qnw, eps)
        k = det_rmsnorm(k, knw, eps)
    pos = np.arange(N) % T
    c = np.asarray(cos, F32)[pos][:, None, :]
    sn = np.asarray(sin, F32)[pos][:, None, :]
    half = hd // 2

    def rope(z):
        return fadd(fmul(z, c), fmul(np.concatenate([-z[..., half:], z[..., :half]], -1), sn))
    qq, qs = quant_sym(rope(q), 127)
    kq, ks = quant_sym(rope(k), 127)
    vq, vs = quant_sym(v, 127)
    i8 = lambda z: z.astype(np.int8)
    return i8(qq), qs, i8(kq), ks, i8(vq), vs


# ------------------------------------------------------------------ attention and log-softmax
P_LEVELS = 16383       # runtime/detrt/qwen3.py:34, 14-bit attention probabilities
MAX_KEYS = 1 << 20     # runtime/detrt/qwen3.py:33


def attention(qq, qs, K, SK, V, SV, start: int, inv_sqrt_hd: float):
    """runtime/detrt/qwen3.py:253-283 for one batch of queries over a key / value cache.

    qq (B, Tq, H, 128) int8 and qs (B, Tq, H) are the queries at positions start .. start+Tq-1;
    K, V (B, S, Hkv, 128) int8 and SK, SV (B, S, Hkv) with S = start + Tq. Returns o (B, Tq, H, 128)
    float32: exact Q K^T, scale chain, causal mask, det_exp, exact row sum, 14-bit P, exact P V."""
    B, Tq, H, _ = qq.shape
    S, Hkv = K.shape[1], K.shape[2]
    rep = H // Hkv
    Kh = np.repeat(K.astype(np.int64), rep, axis=2)               # (B, S, H, 128)
    Vh = np.repeat(V.astype(np.int64), rep, axis=2)
    SKh = np.repeat(np.asarray(SK, F32), rep, axis=2)             # (B, S, H)
    SVh = np.repeat(np.asarray(SV, F32), rep, axis=2)
    dot = np.einsum("bthd,bshd->bhts", qq.astype(np.int64), Kh)   # exact
    qs_ = np.asarray(qs, F32).transpose(0, 2, 1)[..., None]        # (B, H, Tq, 1)
    sk_ = SKh.transpose(0, 2, 1)[:, :, None, :]                    # (B, H, 1, S)
    sc = fmul(fmul(fmul(dot.astype(F32), qs_), sk_), c32(inv_sqrt_hd))
    qpos = start + np.arange(Tq)[:, None]
    sc = np.where(np.arange(S)[None, :] <= qpos, sc, F32(-np.inf)).astype(F32)
    mx = sc.max(axis=-1, keepdims=True)
    e = det_exp(fsub(sc, mx))
    den = exact_rowsum(e, MAX_KEYS)
    Pv = fmul(fdiv(e, den[..., None]), SVh.transpose(0, 2, 1)[:, :, None, :])
    pmax = Pv.max(axis=-1, keepdims=True)
    sp = fdiv(np.maximum(pmax, c32(1e-30)), c32(float(P_LEVELS)))
    pi = np.clip(np.rint(fdiv(Pv, sp)), 0, P_LEVELS).astype(np.int64)
    acc = np.einsum("bhts,bshd->bhtd", pi, Vh)                     # exact in int64
    o = fmul(acc.astype(F32), sp)
    return o.transpose(0, 2, 1, 3)


def det_log(x):
    """runtime/detrt/core.py:130-143: log m as 2 atanh((m-1)/(m+1)) (odd series to s^15), + e ln 2."""
    x = np.asarray(x, F32)
    m, e = np.frexp(x)
    m = fmul(m, c32(2.0))
    ef = (e - 1).astype(F32)
    s = fdiv(fsub(m, c32(1.0)), fadd(m, c32(1.0)))
    s2 = fmul(s, s)
    acc = np.full_like(s, c32(1.0 / 15))
    for k in range(13, 0, -2):
        acc = fadd(fmul(acc, s2), c32(1.0 / k))
    lm = fmul(fmul(acc, s), c32(2.0))
    return fadd(fmul(ef, c32(0.6931471805599453)), lm)


def logprobs(lg):
    """runtime/detrt/qwen3.py:302-312 rows: z = lg - max, z - det_log(exact_rowsum(det_exp(z), 2^18))."""
    lg = np.asarray(lg, F32)
    z = fsub(lg, lg.max(axis=-1, keepdims=True))
    den = exact_rowsum(det_exp(z), 1 << 18)
    return fsub(z, det_log(den)[..., None])


# ------------------------------------------------------------------ the whole forward
def int_gemm(q, Wq):
    """DetLinear.int_gemm on CPU (runtime/detrt/qwen3.py:110-111): q @ Wq^T in float64, exact for
    int8 operands (every partial sum is an integer below 2^53), returned as int64."""
    return (np.asarray(q, np.float64) @ np.asarray(Wq, np.float64).T).astype(np.int64)


def quantize_linear(W, hadamard_block: int):
    """DetLinear's weight quantization (qwen3.py:73-88): (Wq int8, sw float32, bs)."""
    W = np.asarray(W, F32)
    bs = min(hadamard_block, W.shape[1] & -W.shape[1]) if hadamard_block else 0
    Wq, sw = quant_act(W, bs)
    return Wq, sw, bs


def layer_forward(L: dict, x, B: int, T: int, H: int, Hkv: int, eps: float, cos, sin, inv_sqrt_hd: float,
                  qk_norm: bool = True):
    """One decoder layer of DetQwen3.forward for B sequences of T tokens from position 0
    (qwen3.py:239-297): x (B*T, D) float32 -> (B*T, D). L holds float32 norms and quantized
    linears (Wq, sw, bs) under qkv, o, gu, down."""
    Wq, sw, bs = L["qkv"]
    q1, s1 = rmsnorm_quant(x, L["in_norm"], eps, bs)
    qq, qs, kq, ks, vq, vs = qkv_post(int_gemm(q1, Wq), s1, sw, L["q_norm"], L["k_norm"], cos, sin, T, H, Hkv, eps,
                                      qk_norm)
    o = attention(qq.reshape(B, T, H, 128), qs.reshape(B, T, H), kq.reshape(B, T, Hkv, 128), ks.reshape(B, T, Hkv),
                  vq.reshape(B, T, Hkv, 128), vs.reshape(B, T, Hkv), 0, inv_sqrt_hd).reshape(B * T, H * 128)
    Wq, sw, bs = L["o"]
    q2, s2 = quant_act(o, bs)
    r1 = dequant_residual(int_gemm(q2, Wq), s2, sw, x)
    Wq, sw, bs = L["gu"]
    q3, s3 = rmsnorm_quant(r1, L["post_norm"], eps, bs)
    Wq2, sw2, bs2 = L["down"]
    q4, s4 = swiglu_quant(int_gemm(q3, Wq), s3, sw, bs2)
    return dequant_residual(int_gemm(q4, Wq2), s4, sw2, r1)
