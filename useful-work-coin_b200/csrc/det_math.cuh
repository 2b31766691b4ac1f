// detrt's emulated-fp32 math on the GPU, shared by the deterministic-runtime kernels: every
// + - * / sqrt is an explicitly rounded IEEE intrinsic, maxima are exact, and sums are int64 fixed
// point (runtime/detrt/core.py). Used by detq.cu and attn.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

// detrt.core._EXP2 and _LOG2E (core.py:100-102), rounded to float32 as detrt's c32 does.
__constant__ const float kExp2[8] = {(float)1.0, (float)0.6931471824645996, (float)0.2402263879776001,
                            (float)0.055505119264125824, (float)0.00961404386907816, (float)0.001342222560197115,
                            (float)0.0001435537706129253, (float)2.1489791834028438e-05};
constexpr float kLog2e = (float)1.4426950408889634;
constexpr float kTiny = (float)1e-8;

__device__ __forceinline__ float pow2f(int n) { return __int_as_float((n + 127) << 23); }
__device__ __forceinline__ double pow2d(int n) { return __longlong_as_double((long long)(n + 1023) << 52); }

// Integer rounding on the FMA / ALU pipes instead of the conversion unit. Adding 1.5 * 2^23 puts
// an |x| < 2^22 into the binade whose ulp is 1, so the addition itself rounds x to an integer in
// the chosen direction (exactly), and that integer is the low mantissa bits of the sum.
constexpr float kRoundMagic = 12582912.0f;    // 1.5 * 2^23
constexpr int kRoundMagicBits = 0x4B400000;   // its bit pattern
__device__ __forceinline__ float floor_small(float x) { return __fsub_rn(__fadd_rd(x, kRoundMagic), kRoundMagic); }
__device__ __forceinline__ int floor_small_int(float x) { return __float_as_int(__fadd_rd(x, kRoundMagic)) - kRoundMagicBits; }
__device__ __forceinline__ float rint_small(float x) { return __fsub_rn(__fadd_rn(x, kRoundMagic), kRoundMagic); }
// an integer-valued |x| < 2^22 as int
__device__ __forceinline__ int int_of_small(float x) { return __float_as_int(__fadd_rn(x, kRoundMagic)) - kRoundMagicBits; }
// float(d) for |d| < 2^22 (exact: no rounding happens)
__device__ __forceinline__ float float_of_small(int d) { return __fsub_rn(__int_as_float(kRoundMagicBits + d), kRoundMagic); }

// detrt.core.det_exp (core.py:111-127): 2^(z log2 e) as 2^n * poly(f), one rounding per op.
// After the range clamp |t| < 128, so floor(t) comes from floor_small.
__device__ __forceinline__ float det_exp(float z) {
  float t = __fmul_rn(z, kLog2e);
  const bool under = t < -126.0f, over = t >= 128.0f;
  if (under || over || isnan(t)) t = 0.0f;
  const float n = floor_small(t);
  const float f = __fsub_rn(t, n);
  float p = kExp2[7];
#pragma unroll
  for (int i = 6; i >= 0; i--) p = __fadd_rn(__fmul_rn(p, f), kExp2[i]);
  float r = __fmul_rn(p, pow2f(floor_small_int(t)));
  if (under) r = 0.0f;
  if (over) r = __int_as_float(0x7f800000);
  if (isnan(z)) r = z;
  return r;
}

__device__ __forceinline__ float deq(int acc, float s, float sw) { return __fmul_rn(__fmul_rn(__int2float_rn(acc), s), sw); }

// detgpu's SwiGLU element (kernels.py:356-396): fmul(g / (1 + det_exp(-g)), u), one rounding per op.
__device__ __forceinline__ float det_swiglu(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, det_exp(-g))), u);
}

__device__ __forceinline__ float warp_maxf(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ long long warp_sumll(long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide max / int64 sum over the CTA's NT threads (exact, any order).
template <int NT>
__device__ float block_maxf(float v, float* red) {
  v = warp_maxf(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int i = 1; i < NT / 32; i++) m = fmaxf(m, red[i]);
  return m;
}
template <int NT>
__device__ long long block_sumll(long long v, long long* red) {
  v = warp_sumll(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  long long s = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; i++) s += red[i];
  return s;
}

}  // namespace
