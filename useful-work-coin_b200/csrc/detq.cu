// Producers and consumers of the deterministic int8 linear (runtime/detrt, runtime/detgpu), sm_100a.
//
// Each kernel reproduces detrt's emulated-fp32 arithmetic bit for bit: every + - * / sqrt is an
// explicitly rounded IEEE intrinsic (__fadd_rn, __fmul_rn, __fdiv_rn, __fsqrt_rn), which the
// compiler never contracts, applied in detrt's order; maxima are exact and sums are detrt's int64
// fixed point, so neither depends on how threads split a row.
//
//   quant_act         fwht(bs) + quant_sym(64) + 1/sqrt(bs) scale fold   runtime/detrt/core.py:171-196
//   quant_rows_had    the same from bf16 rows (the mined bf16 linear)      miner/ampere/uwc_ampere/kernels.cu:717-778
//   fwht_absmax /     the row-parallel split of quant_act: per-shard max,  (tensor-parallel form, new)
//   quant_act_global  then quantize with the max over shards
//   rmsnorm_quant     det_rmsnorm then quant_act                           runtime/detgpu/kernels.py:117-191
//   swiglu_quant      quant_act(det_silu(gate) * up) of the dequantized    runtime/detgpu/kernels.py:356-396
//                     gate/up GEMM output
//   swiglu            the fp32 fmul(det_silu(gate), up) row (tensor-parallel form, new)
//   dequant_residual  x + fmul(fmul(float(acc), s), sw)                    runtime/detgpu/kernels.py:346-354
//   qkv_post          dequant, q/k head RMSNorm, rope, quant_sym(127)      runtime/detgpu/kernels.py:303-344
//
// Row kernels keep one row in shared memory (one CTA of 256 threads per row) and read / write HBM
// once; they are bandwidth-bound by design.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <set>
#include <utility>

#include "det_math.cuh"
#include "uwc_device.cuh"
#include "uwc_host.h"
#include "uwc_tp.cuh"

namespace {

constexpr int kRowThreads = 256;      // threads per row CTA (1024 for few-row calls)
constexpr int kMaxRowSmem = 200 * 1024;   // k <= 51200 floats per row

// One bs = 32 E block per warp, E consecutive elements per lane in registers: stages h < E pair
// elements of a lane, stages h >= E pair lane l with lane l ^ (h / E) (the lower lane keeps a + b,
// the upper a - b, a the lower element): the same pairs, operands and roundings as the staged
// transform below.
template <int E>
__device__ __forceinline__ void fwht_block_lane(float* blk) {
  const int lane = threadIdx.x & 31;
  float v[E];
  float* p = blk + E * lane;
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int i = 0; i < E / 4; i++) {
      const float4 x = reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; i++) v[i] = p[i];
  }
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int i = 0; i < E; i++) {
      if (i & h) continue;
      const float a = v[i], b = v[i + h];
      v[i] = __fadd_rn(a, b);
      v[i + h] = __fsub_rn(a, b);
    }
  }
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const bool upper = lane & d;
#pragma unroll
    for (int i = 0; i < E; i++) {
      const float o = __shfl_xor_sync(0xffffffffu, v[i], d);
      v[i] = upper ? __fsub_rn(o, v[i]) : __fadd_rn(v[i], o);
    }
  }
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int i = 0; i < E / 4; i++)
      reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < E; i++) p[i] = v[i];
  }
}

template <int NT, int E>
__device__ void fwht_row_warp(float* row, int k) {
  const int nblk = k / (32 * E);
  for (int blk = threadIdx.x >> 5; blk < nblk; blk += NT / 32) fwht_block_lane<E>(row + (size_t)blk * 32 * E);
  __syncthreads();
}

// In-place unnormalized block Walsh-Hadamard transform of a shared-memory row (core.py:171-185):
// stages h = 1, 2, 4, ... < bs, pairs (i, i + h) of each 2h-block -> (a + b, a - b). Blocks of 32
// to 512 elements run one per warp in registers (fwht_block_lane), others staged in shared memory.
template <int NT>
__device__ void fwht_row(float* row, int k, int bs) {
  switch (bs) {
    case 512: fwht_row_warp<NT, 16>(row, k); return;
    case 256: fwht_row_warp<NT, 8>(row, k); return;
    case 128: fwht_row_warp<NT, 4>(row, k); return;
    case 64: fwht_row_warp<NT, 2>(row, k); return;
    case 32: fwht_row_warp<NT, 1>(row, k); return;
    default: break;
  }
  for (int lh = 0; (1 << lh) < bs; lh++) {
    const int h = 1 << lh;
    for (int p = threadIdx.x; p < (k >> 1); p += NT) {
      const int i = ((p >> lh) << (lh + 1)) | (p & (h - 1)), j = i + h;
      const float a = row[i], b = row[j];
      row[i] = __fadd_rn(a, b);
      row[j] = __fsub_rn(a, b);
    }
    __syncthreads();
  }
}

// quant_sym of the staged row with row absmax `amax` and qmax = 64 (core.py:162-168), then the
// quant_act scale fold (core.py:188-196).
template <int NT>
__device__ void quant_row64(const float* row, int k, int bs, float amax, int8_t* q, float* scale_out) {
  const float s = __fdiv_rn(fmaxf(amax, kTiny), 64.0f);
  for (int i = threadIdx.x * 4; i < k; i += NT * 4) {
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      // |row / s| <= 64 (1 + 2^-22): rint_small and int_of_small are exact here
      const float v = fminf(fmaxf(rint_small(__fdiv_rn(row[i + j], s)), -64.f), 64.f);
      o |= ((uint32_t)(uint8_t)(int8_t)int_of_small(v)) << (8 * j);
    }
    *reinterpret_cast<uint32_t*>(q + i) = o;
  }
  if (threadIdx.x == 0) *scale_out = bs > 1 ? __fmul_rn(s, __fdiv_rn(1.0f, __fsqrt_rn((float)bs))) : s;
}

// k % 4 == 0 (every caller checks): four elements per thread and step
template <int NT>
__device__ float row_absmax(const float* row, int k, float* red) {
  float mx = 0.f;
  for (int i = 4 * threadIdx.x; i < k; i += 4 * NT) {
    const float4 v = *reinterpret_cast<const float4*>(row + i);
    mx = fmaxf(fmaxf(mx, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
  }
  return block_maxf<NT>(mx, red);
}

// Stage row r of x (fp32 or bf16, k % 4 == 0) into shared memory.
template <int NT, bool BF16>
__device__ void load_row(const void* x, int r, int k, float* row) {
  if (BF16) {
    const uint2* src = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + (uint64_t)r * k);
    for (int i = threadIdx.x; i < k / 4; i += NT) {
      const uint2 v = src[i];
      row[4 * i] = __uint_as_float(v.x << 16);
      row[4 * i + 1] = __uint_as_float(v.x & 0xFFFF0000u);
      row[4 * i + 2] = __uint_as_float(v.y << 16);
      row[4 * i + 3] = __uint_as_float(v.y & 0xFFFF0000u);
    }
  } else {
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(x) + (uint64_t)r * k);
    for (int i = threadIdx.x; i < k / 4; i += NT) reinterpret_cast<float4*>(row)[i] = src[i];
  }
  __syncthreads();
}

// MODE 0: quant_act (local absmax). MODE 1: only the transformed row's absmax -> amax[r].
// MODE 2: quantize with amax[r] given (the max over the row's column shards).
template <int NT, int MODE, bool BF16>
__global__ void __launch_bounds__(NT) k_quant_act(const void* __restrict__ x, int k, int bs,
                                                           float* __restrict__ amax, int8_t* __restrict__ q,
                                                           float* __restrict__ scale) {
  extern __shared__ float row[];
  // Launched early behind the previous kernel: wait for its writes, then let a weight-streaming GEMM
  // behind this kernel start fetching its weights. The bf16 form also quantizes weights, so it
  // never lets its successor start early.
  pdl_wait();
  if (!BF16) pdl_trigger();
  __shared__ float red[NT / 32];
  const int r = blockIdx.x;
  load_row<NT, BF16>(x, r, k, row);
  if (bs > 1) fwht_row<NT>(row, k, bs);
  if (MODE == 2) {
    quant_row64<NT>(row, k, bs, amax[r], q + (uint64_t)r * k, scale + r);
    return;
  }
  const float mx = row_absmax<NT>(row, k, red);
  if (MODE == 1) {
    if (threadIdx.x == 0) amax[r] = mx;
    return;
  }
  quant_row64<NT>(row, k, bs, mx, q + (uint64_t)r * k, scale + r);
}

// quant_act of a row-parallel shard with the whole row's absmax, exchanged in the kernel: each CTA
// (one row) stores its shard's absmax, tagged with the call's epoch, into every rank's exchange
// buffer, polls for every rank's value of the row, and quantizes with the maximum (the fwht_absmax, MAX
// all-reduce and quant_act_global sequence: the same maximum, so the same bits).
template <int NT>
__global__ void __launch_bounds__(NT) k_quant_act_tp(const float* __restrict__ x, int k, int bs,
                                                     int8_t* __restrict__ q, float* __restrict__ scale, TPArgs tp,
                                                     uint32_t* status, uint64_t wait_ns) {
  extern __shared__ float row[];
  __shared__ float red[NT / 32];
  __shared__ float src_max[uwc_tp::kMaxWorld];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  uint8_t* const mine = tp.base[tp.rank];
  const uint64_t E = uwc_tp::call_epoch(mine);
  const int par = (int)(E & 1);
  load_row<NT, false>(x, r, k, row);
  if (bs > 1) fwht_row<NT>(row, k, bs);
  const float mx = row_absmax<NT>(row, k, red);
  const int p = threadIdx.x;
  if (p < tp.world) {
    uwc_tp::st_sys(uwc_tp::amax_slot(tp.base[p], tp.L, par, tp.rank, r), uwc_tp::tagged(E, __float_as_uint(mx)));
    bool ok = true;
    const uint32_t v = uwc_tp::wait_tagged(uwc_tp::amax_slot(mine, tp.L, par, p, r), E, uwc_tp::now_ns() + wait_ns,
                                           status, &ok);
    src_max[p] = ok ? __uint_as_float(v) : mx;
  }
  __syncthreads();
  float am = src_max[0];
  for (int i = 1; i < tp.world; i++) am = fmaxf(am, src_max[i]);
  quant_row64<NT>(row, k, bs, am, q + (uint64_t)r * k, scale + r);
  __syncthreads();
  if (threadIdx.x == 0) uwc_tp::call_end(mine, E, gridDim.x);
}

// det_rmsnorm (core.py:151-159, exact_rowsum core.py:85-108) then quant_act.
template <int NT>
__global__ void __launch_bounds__(NT) k_rmsnorm_quant(const float* __restrict__ x, const float* __restrict__ w,
                                                               int k, int bs, float inv_d, float eps, int L,
                                                               int8_t* __restrict__ q, float* __restrict__ scale) {
  extern __shared__ float row[];
  pdl_wait();      // launched early behind the previous kernel: its writes are visible from here
  pdl_trigger();   // a weight-streaming GEMM behind this kernel may start fetching its weights
  __shared__ float red[NT / 32];
  __shared__ long long redl[NT / 32];
  const int r = blockIdx.x;
  load_row<NT, false>(x, r, k, row);
  // four elements per thread and step (k % 4 == 0)
  float mx = 0.f;
  for (int i = 4 * threadIdx.x; i < k; i += 4 * NT) {
    const float4 v = *reinterpret_cast<const float4*>(row + i);
    mx = fmaxf(fmaxf(mx, fmaxf(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y))),
               fmaxf(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w)));
  }
  mx = block_maxf<NT>(mx, red);
  int e;
  frexpf(mx, &e);
  const int sh = min(max((62 - L) - e, -1000), 1000);
  const double up = pow2d(sh);
  long long acc = 0;
  for (int i = 4 * threadIdx.x; i < k; i += 4 * NT) {
    const float4 v = *reinterpret_cast<const float4*>(row + i);
    acc += __double2ll_rn((double)__fmul_rn(v.x, v.x) * up) + __double2ll_rn((double)__fmul_rn(v.y, v.y) * up) +
           __double2ll_rn((double)__fmul_rn(v.z, v.z) * up) + __double2ll_rn((double)__fmul_rn(v.w, v.w) * up);
  }
  acc = block_sumll<NT>(acc, redl);
  const float ss = __double2float_rn(__ll2double_rn(acc) * pow2d(-sh));
  const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, inv_d), eps)));
  for (int i = 4 * threadIdx.x; i < k; i += 4 * NT) {
    float4 v = *reinterpret_cast<const float4*>(row + i);
    const float4 wv = __ldg(reinterpret_cast<const float4*>(w + i));
    v.x = __fmul_rn(__fmul_rn(v.x, rr), wv.x);
    v.y = __fmul_rn(__fmul_rn(v.y, rr), wv.y);
    v.z = __fmul_rn(__fmul_rn(v.z, rr), wv.z);
    v.w = __fmul_rn(__fmul_rn(v.w, rr), wv.w);
    *reinterpret_cast<float4*>(row + i) = v;
  }
  __syncthreads();
  if (bs > 1) fwht_row<NT>(row, k, bs);
  const float am = row_absmax<NT>(row, k, red);
  quant_row64<NT>(row, k, bs, am, q + (uint64_t)r * k, scale + r);
}

// Rows with 512-element Hadamard blocks (any number of rows): warp w holds block w of the row in registers,
// 16 consecutive elements per lane, from the global load to the int8 store; only the block maxima
// and fixed-point sums pass through shared memory. The transform is fwht_block_lane's stages on the
// registers, and every other operation is the staged kernels' in the same order: the same bits.
// RMS = false is quant_act (k_quant_act MODE 0), RMS = true rmsnorm_quant. blockDim = 32 (k / 512).
// TP: the row-parallel form (k_quant_act_tp): the shard's absmax is exchanged with every rank and
// the row is quantized with the maximum.
__device__ __forceinline__ float cta_maxf(float v, float* red) {
  v = warp_maxf(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, red[i]);
  return m;
}
__device__ __forceinline__ long long cta_sumll(long long v, long long* red) {
  v = warp_sumll(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  long long t = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
  return t;
}

// The plain form is held to 32 registers so that two rows' CTAs share an SM when there are many
// rows (16384 rows of k = 14336: 500 -> 426 us).
template <bool RMS, bool TP>
__global__ void __launch_bounds__(1024, RMS || TP ? 1 : 2) k_row_quant512(const float* __restrict__ x, const float* __restrict__ w, int k,
                                                       float inv_d, float eps, int L, int8_t* __restrict__ q,
                                                       float* __restrict__ scale, TPArgs tp, uint32_t* status,
                                                       uint64_t wait_ns) {
  __shared__ float redf[32];
  __shared__ long long redl[32];
  __shared__ float src_max[uwc_tp::kMaxWorld];
  pdl_wait();      // launched early behind the previous kernel: its writes are visible from here
  pdl_trigger();   // a weight-streaming GEMM behind this kernel may start fetching its weights
  const int r = blockIdx.x, lane = threadIdx.x & 31;
  const size_t off = (size_t)(threadIdx.x >> 5) * 512 + lane * 16;
  float v[16];
  {
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)r * k + off);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 a = src[i];
      v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
    }
  }
  if (RMS) {
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) mx = fmaxf(mx, __fmul_rn(v[i], v[i]));
    mx = cta_maxf(mx, redf);
    int e;
    frexpf(mx, &e);
    const int sh = min(max((62 - L) - e, -1000), 1000);
    const double up = pow2d(sh);
    long long acc = 0;
#pragma unroll
    for (int i = 0; i < 16; i++) acc += __double2ll_rn((double)__fmul_rn(v[i], v[i]) * up);
    acc = cta_sumll(acc, redl);
    const float ss = __double2float_rn(__ll2double_rn(acc) * pow2d(-sh));
    const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, inv_d), eps)));
    const float4* wp = reinterpret_cast<const float4*>(w + off);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 wv = __ldg(wp + i);
      v[4 * i] = __fmul_rn(__fmul_rn(v[4 * i], rr), wv.x);
      v[4 * i + 1] = __fmul_rn(__fmul_rn(v[4 * i + 1], rr), wv.y);
      v[4 * i + 2] = __fmul_rn(__fmul_rn(v[4 * i + 2], rr), wv.z);
      v[4 * i + 3] = __fmul_rn(__fmul_rn(v[4 * i + 3], rr), wv.w);
    }
  }
  // fwht_block_lane<16> on registers: stages inside the lane, then across lanes
#pragma unroll
  for (int h = 1; h < 16; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 16; i++) {
      if (i & h) continue;
      const float a = v[i], b = v[i + h];
      v[i] = __fadd_rn(a, b);
      v[i + h] = __fsub_rn(a, b);
    }
  }
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const bool upper = lane & d;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float o = __shfl_xor_sync(0xffffffffu, v[i], d);
      v[i] = upper ? __fsub_rn(o, v[i]) : __fadd_rn(v[i], o);
    }
  }
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < 16; i++) am = fmaxf(am, fabsf(v[i]));
  am = cta_maxf(am, redf);
  uint64_t E = 0;
  if (TP) {
    uint8_t* const mine = tp.base[tp.rank];
    E = uwc_tp::call_epoch(mine);
    const int par = (int)(E & 1), p = threadIdx.x;
    if (p < tp.world) {
      uwc_tp::st_sys(uwc_tp::amax_slot(tp.base[p], tp.L, par, tp.rank, r), uwc_tp::tagged(E, __float_as_uint(am)));
      bool ok = true;
      const uint32_t got = uwc_tp::wait_tagged(uwc_tp::amax_slot(mine, tp.L, par, p, r), E,
                                               uwc_tp::now_ns() + wait_ns, status, &ok);
      src_max[p] = ok ? __uint_as_float(got) : am;
    }
    __syncthreads();
    for (int i = 0; i < tp.world; i++) am = fmaxf(am, src_max[i]);
  }
  // quant_row64: q = clamp(rint(v / s), -64, 64), s = max(amax, tiny) / 64
  const float s = __fdiv_rn(fmaxf(am, kTiny), 64.0f);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float t = fminf(fmaxf(rint_small(__fdiv_rn(v[4 * i + j], s)), -64.f), 64.f);
      word |= ((uint32_t)(uint8_t)(int8_t)int_of_small(t)) << (8 * j);
    }
    o[i] = word;
  }
  *reinterpret_cast<uint4*>(q + (size_t)r * k + off) = make_uint4(o[0], o[1], o[2], o[3]);
  if (threadIdx.x == 0) scale[r] = __fmul_rn(s, __fdiv_rn(1.0f, __fsqrt_rn(512.0f)));
  if (TP) {
    __syncthreads();
    if (threadIdx.x == 0) uwc_tp::call_end(tp.base[tp.rank], E, gridDim.x);
  }
}

// fmul(det_silu(gate), up) of the dequantized gate/up GEMM output (N x 2I int32)
__device__ __forceinline__ float swiglu_at(const int32_t* ar, float s, const float* sw, int I, int i) {
  return det_swiglu(deq(ar[i], s, sw[i]), deq(ar[I + i], s, sw[I + i]));
}

// quant_act(fmul(det_silu(gate), up)) of the gate/up GEMM output, one row per CTA.
template <int NT>
__global__ void __launch_bounds__(NT) k_swiglu_quant(const int32_t* __restrict__ acc,
                                                              const float* __restrict__ s3, const float* __restrict__ sw,
                                                              int I, int bs, int8_t* __restrict__ q,
                                                              float* __restrict__ scale) {
  extern __shared__ float row[];
  pdl_wait();      // launched early behind the previous kernel: its writes are visible from here
  pdl_trigger();   // a weight-streaming GEMM behind this kernel may start fetching its weights
  __shared__ float red[NT / 32];
  const int r = blockIdx.x;
  const float s = s3[r];
  const int32_t* ar = acc + (uint64_t)r * 2 * I;
  // four elements per thread and step (I % 4 == 0): 16-byte loads of the gate and up halves
  for (int i = 4 * threadIdx.x; i < I; i += 4 * NT) {
    const int4 g4 = __ldg(reinterpret_cast<const int4*>(ar + i)), u4 = __ldg(reinterpret_cast<const int4*>(ar + I + i));
    const float4 sg = __ldg(reinterpret_cast<const float4*>(sw + i)), su = __ldg(reinterpret_cast<const float4*>(sw + I + i));
    const int gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
    const float sgv[4] = {sg.x, sg.y, sg.z, sg.w}, suv[4] = {su.x, su.y, su.z, su.w};
    float o[4];
#pragma unroll
    for (int x = 0; x < 4; x++) {
      const float g = deq(gv[x], s, sgv[x]), u = deq(uv[x], s, suv[x]);
      o[x] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, det_exp(-g))), u);
    }
    *reinterpret_cast<float4*>(row + i) = make_float4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (bs > 1) fwht_row<NT>(row, I, bs);
  const float am = row_absmax<NT>(row, I, red);
  quant_row64<NT>(row, I, bs, am, q + (uint64_t)r * I, scale + r);
}

// The fp32 SwiGLU row alone (the input of a row-parallel down projection, quantized per shard).
__global__ void k_swiglu(const int32_t* __restrict__ acc, const float* __restrict__ s3, const float* __restrict__ sw,
                         int I, float* __restrict__ h) {
  const int r = blockIdx.y;
  const int32_t* ar = acc + (uint64_t)r * 2 * I;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < I; i += gridDim.x * blockDim.x)
    h[(uint64_t)r * I + i] = swiglu_at(ar, s3[r], sw, I, i);
}

// out = fadd(x, deq(acc)) (x == nullptr: out = deq(acc)), 4 elements per thread (k % 4 == 0).
__global__ void k_dequant_residual(const int32_t* __restrict__ acc, const float* __restrict__ s,
                                   const float* __restrict__ sw, const float* __restrict__ x, int k, uint64_t n4,
                                   float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t e = 4 * i, r = e / k;
    const int c = (int)(e - r * k);
    const int4 a = reinterpret_cast<const int4*>(acc)[i];
    const float4 w = *reinterpret_cast<const float4*>(sw + c);
    const float sr = s[r];
    float4 o = make_float4(deq(a.x, sr, w.x), deq(a.y, sr, w.y), deq(a.z, sr, w.z), deq(a.w, sr, w.w));
    if (x) {
      const float4 xv = reinterpret_cast<const float4*>(x)[i];
      o = make_float4(__fadd_rn(xv.x, o.x), __fadd_rn(xv.y, o.y), __fadd_rn(xv.z, o.z), __fadd_rn(xv.w, o.w));
    }
    reinterpret_cast<float4*>(out)[i] = o;
  }
}

// quant_sym(qmax = 127) of one 128-wide head held as element lane + 32 j in v[j].
__device__ __forceinline__ void head_quant127(const float* v, int lane, int8_t* q, float* scale) {
  float mx = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++) mx = fmaxf(mx, fabsf(v[j]));
  mx = warp_maxf(mx);
  const float s = __fdiv_rn(fmaxf(mx, kTiny), 127.0f);
#pragma unroll
  for (int j = 0; j < 4; j++) q[lane + 32 * j] = (int8_t)(int)fminf(fmaxf(rintf(__fdiv_rn(v[j], s)), -127.f), 127.f);
  if (lane == 0) *scale = s;
}

// The qkv GEMM's int32 row -> quantized q, k, v heads (detrt/fast.py:108-120). One CTA per row
// (token), one warp per head; element i of a head is v[j] of lane i % 32 with j = i / 32, so the
// rope partner i +- 64 is v[j +- 2] of the same lane.
// The KV cache a decode step's keys and values go straight into (uwc_qkv_post_kv): (B, Hkv, maxlen,
// 128) int8 rows and (B, Hkv, maxlen) scales; k == nullptr: write the kq / vq rows instead.
struct KVDest {
  int8_t* k;
  float* sk;
  int8_t* v;
  float* sv;
  int maxlen;
};

__global__ void __launch_bounds__(kRowThreads) k_qkv_post(
    const int32_t* __restrict__ acc, const float* __restrict__ s1, const float* __restrict__ sw,
    const float* __restrict__ qnw, const float* __restrict__ knw, const float* __restrict__ cosT,
    const float* __restrict__ sinT, int T, int H, int Hkv, float inv_hd, float eps, int qknorm,
    int8_t* __restrict__ qq, float* __restrict__ qs, int8_t* __restrict__ kq, float* __restrict__ ks,
    int8_t* __restrict__ vq, float* __restrict__ vs, const int* __restrict__ pos0, const KVDest kv) {
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // with a cache destination: token row % T of sequence row / T lands at position pos0 + row % T
  const int cpos = kv.k ? __ldg(pos0) + row % T : 0;
  const long long cbase = kv.k ? (long long)(row / T) * Hkv * kv.maxlen + cpos : 0;   // (b, head 0, cpos)
  // rope table row: position r % T, offset by a device-side start position when given
  const int nh = H + 2 * Hkv, width = nh * 128, t = row % T + (pos0 ? __ldg(pos0) : 0);
  const float s = s1[row];
  for (int hh = warp; hh < nh; hh += kRowThreads / 32) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int c = hh * 128 + lane + 32 * j;
      v[j] = deq(acc[(uint64_t)row * width + c], s, sw[c]);
    }
    if (hh >= H + Hkv) {
      const int hv = hh - H - Hkv;
      if (!kv.k) {
        head_quant127(v, lane, vq + ((uint64_t)row * Hkv + hv) * 128, vs + (uint64_t)row * Hkv + hv);
      } else if (cpos < kv.maxlen) {
        const long long d = cbase + (long long)hv * kv.maxlen;
        head_quant127(v, lane, kv.v + d * 128, kv.sv + d);
      }
      continue;
    }
    if (qknorm) {
      // det_rmsnorm over the head (exact_rowsum with max_terms = 128, so L = 7)
      float mx = 0.f;
#pragma unroll
      for (int j = 0; j < 4; j++) mx = fmaxf(mx, __fmul_rn(v[j], v[j]));
      mx = warp_maxf(mx);
      int e;
      frexpf(mx, &e);
      const int sh = min(max((62 - 7) - e, -1000), 1000);
      long long a = 0;
#pragma unroll
      for (int j = 0; j < 4; j++) a += __double2ll_rn((double)__fmul_rn(v[j], v[j]) * pow2d(sh));
      a = warp_sumll(a);
      const float ss = __double2float_rn(__ll2double_rn(a) * pow2d(-sh));
      const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, inv_hd), eps)));
      const float* w = hh < H ? qnw : knw;
#pragma unroll
      for (int j = 0; j < 4; j++) v[j] = __fmul_rn(__fmul_rn(v[j], rr), w[lane + 32 * j]);
    }
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int i = lane + 32 * j;
      const float rot = j < 2 ? -v[j + 2] : v[j - 2];
      o[j] = __fadd_rn(__fmul_rn(v[j], cosT[t * 128 + i]), __fmul_rn(rot, sinT[t * 128 + i]));
    }
    if (hh < H) {
      head_quant127(o, lane, qq + ((uint64_t)row * H + hh) * 128, qs + (uint64_t)row * H + hh);
    } else if (!kv.k) {
      head_quant127(o, lane, kq + ((uint64_t)row * Hkv + hh - H) * 128, ks + (uint64_t)row * Hkv + hh - H);
    } else if (cpos < kv.maxlen) {
      const long long d = cbase + (long long)(hh - H) * kv.maxlen;
      head_quant127(o, lane, kv.k + d * 128, kv.sk + d);
    }
  }
}

// smallest L >= 1 with 2^L >= n (detrt's ceil(log2(max_terms)))
int ceil_log2(int n) {
  int L = 1;
  while ((1 << L) < n) L++;
  return L;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// Row kernels stage a row in dynamic shared memory; rows over 48 KiB need the opt-in, set once per
// kernel and device (never during a stream capture after the first call).
int row_smem_ok(int k, const void* kernel) {
  if (4 * k > kMaxRowSmem) return UWC_ERR_SHAPE;
  if (4 * k <= 48 * 1024) return UWC_OK;
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({dev, kernel})) return UWC_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxRowSmem) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  done.insert({dev, kernel});
  return UWC_OK;
}

// Fewer rows than SMs (decode): 1024 threads per row shorten each row's latency.
bool few_rows(int m) { return m < uwc_num_sms(); }

// The register-resident few-row kernels: 512-element Hadamard blocks, one warp each, at most 32.
bool reg_row(int k, int bs) { return bs == 512 && k % 512 == 0 && k <= 32 * 512; }

bool bs_ok(int k, int bs) { return bs <= 1 || ((bs & (bs - 1)) == 0 && k % bs == 0); }

std::atomic<int> g_row_pdl{1};

// Launches a few-row kernel with programmatic stream serialization: it is scheduled while the
// previous kernel of the stream finishes and waits for it (pdl_wait) before touching memory.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), int grid, int threads, size_t smem, void* stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_row_pdl.load();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  uwc_count_launch();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  return uwc_launch_status();
}

template <int MODE, bool BF16>
int launch_quant(const void* x, int m, int k, int bs, float* amax, int8_t* q, float* scale, void* stream) {
  if (!x || m < 0 || k <= 0 || k % 4 || !bs_ok(k, bs)) return UWC_ERR_ARG;
  if (MODE != 1 && (!q || !scale)) return UWC_ERR_ARG;
  if (MODE != 0 && !amax) return UWC_ERR_ARG;
  if (!aligned16(x) || (q && ((uintptr_t)q & 3))) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  if (m == 0) return UWC_OK;
  if (MODE == 0 && !BF16 && reg_row(k, bs) && aligned16(q))
    return launch_pdl(k_row_quant512<false, false>, m, 32 * (k / 512), 0, stream, static_cast<const float*>(x),
                      static_cast<const float*>(nullptr), k, 0.f, 0.f, 0, q, scale, TPArgs{},
                      static_cast<uint32_t*>(nullptr), (uint64_t)0);
  if (few_rows(m)) {
    const int rc = row_smem_ok(k, (const void*)k_quant_act<1024, MODE, BF16>);
    if (rc != UWC_OK) return rc;
    return launch_pdl(k_quant_act<1024, MODE, BF16>, m, 1024, 4 * k, stream, x, k, bs, amax, q, scale);
  } else {
    const int rc = row_smem_ok(k, (const void*)k_quant_act<kRowThreads, MODE, BF16>);
    if (rc != UWC_OK) return rc;
    k_quant_act<kRowThreads, MODE, BF16><<<m, kRowThreads, 4 * k, (cudaStream_t)stream>>>(x, k, bs, amax, q, scale);
    uwc_count_launch();
  }
  return uwc_launch_status();
}

}  // namespace

void uwc_row_set_pdl(int on) { g_row_pdl.store(on ? 1 : 0); }

extern "C" int uwc_quant_act(const float* x, int m, int k, int bs, int8_t* q, float* scale, void* stream) {
  return launch_quant<0, false>(x, m, k, bs, nullptr, q, scale, stream);
}

extern "C" int uwc_quant_rows_had(const uint16_t* x_bf16, int m, int k, int bs, int8_t* q, float* scale, void* stream) {
  return launch_quant<0, true>(x_bf16, m, k, bs, nullptr, q, scale, stream);
}

extern "C" int uwc_fwht_absmax(const float* x, int m, int k, int bs, float* amax, void* stream) {
  return launch_quant<1, false>(x, m, k, bs, amax, nullptr, nullptr, stream);
}

extern "C" int uwc_quant_act_global(const float* x, int m, int k, int bs, const float* amax, int8_t* q, float* scale,
                                    void* stream) {
  return launch_quant<2, false>(x, m, k, bs, const_cast<float*>(amax), q, scale, stream);
}

extern "C" int uwc_quant_act_tp(const float* x, int m, int k, int bs, int8_t* q, float* scale, const UwcTP* tp,
                                void* stream) {
  if (!x || !q || !scale || m < 0 || k <= 0 || k % 4 || !bs_ok(k, bs)) return UWC_ERR_ARG;
  if (!aligned16(x) || ((uintptr_t)q & 3)) return UWC_ERR_ALIGN;
  TPArgs args;
  const int rc = uwc_tp_args(tp, m, 0, &args);
  if (rc != UWC_OK) return rc;
  UWC_CHECK_DEVICE();
  if (m == 0) return UWC_OK;
  // one CTA per row, all resident (the rows wait for the peers' rows)
  if (m > uwc_num_sms()) return UWC_ERR_SHAPE;
  const uint64_t wns = uwc_wait_ns() ? uwc_wait_ns() : uwc_tp::kWaitNs;
  if (reg_row(k, bs) && aligned16(q))
    return launch_pdl(k_row_quant512<false, true>, m, 32 * (k / 512), 0, stream, x, static_cast<const float*>(nullptr),
                      k, 0.f, 0.f, 0, q, scale, args, uwc_status_ptr(), wns);
  const int rs = row_smem_ok(k, (const void*)k_quant_act_tp<1024>);
  if (rs != UWC_OK) return rs;
  const uint64_t ns = uwc_wait_ns();
  return launch_pdl(k_quant_act_tp<1024>, m, 1024, 4 * k, stream, x, k, bs, q, scale, args, uwc_status_ptr(),
                    ns ? ns : uwc_tp::kWaitNs);
}

extern "C" int uwc_rmsnorm_quant(const float* x, const float* w, int m, int k, int bs, double eps, int8_t* q,
                                 float* scale, void* stream) {
  if (!x || !w || !q || !scale || m < 0 || k <= 0 || k % 4 || !bs_ok(k, bs)) return UWC_ERR_ARG;
  if (!aligned16(x) || !aligned16(w) || ((uintptr_t)q & 3)) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  if (m == 0) return UWC_OK;
  // detrt rounds 1/d and eps from float64 to float32 (core.c32)
  const float inv_d = (float)(1.0 / k), eps32 = (float)eps;
  if (reg_row(k, bs) && aligned16(q))
    return launch_pdl(k_row_quant512<true, false>, m, 32 * (k / 512), 0, stream, x, w, k, inv_d, eps32, ceil_log2(k),
                      q, scale, TPArgs{}, static_cast<uint32_t*>(nullptr), (uint64_t)0);
  if (few_rows(m)) {
    const int rc = row_smem_ok(k, (const void*)k_rmsnorm_quant<1024>);
    if (rc != UWC_OK) return rc;
    return launch_pdl(k_rmsnorm_quant<1024>, m, 1024, 4 * k, stream, x, w, k, bs, inv_d, eps32, ceil_log2(k), q,
                      scale);
  } else {
    const int rc = row_smem_ok(k, (const void*)k_rmsnorm_quant<kRowThreads>);
    if (rc != UWC_OK) return rc;
    k_rmsnorm_quant<kRowThreads><<<m, kRowThreads, 4 * k, (cudaStream_t)stream>>>(x, w, k, bs, inv_d, eps32,
                                                                                 ceil_log2(k), q, scale);
    uwc_count_launch();
  }
  return uwc_launch_status();
}

extern "C" int uwc_swiglu_quant(const int32_t* acc, const float* s3, const float* sw, int m, int I, int bs, int8_t* q,
                                float* scale, void* stream) {
  if (!acc || !s3 || !sw || !q || !scale || m < 0 || I <= 0 || I % 4 || !bs_ok(I, bs)) return UWC_ERR_ARG;
  if (((uintptr_t)q & 3) || !aligned16(acc) || !aligned16(sw)) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  if (m == 0) return UWC_OK;
  if (few_rows(m)) {
    const int rc = row_smem_ok(I, (const void*)k_swiglu_quant<1024>);
    if (rc != UWC_OK) return rc;
    return launch_pdl(k_swiglu_quant<1024>, m, 1024, 4 * I, stream, acc, s3, sw, I, bs, q, scale);
  } else {
    const int rc = row_smem_ok(I, (const void*)k_swiglu_quant<kRowThreads>);
    if (rc != UWC_OK) return rc;
    k_swiglu_quant<kRowThreads><<<m, kRowThreads, 4 * I, (cudaStream_t)stream>>>(acc, s3, sw, I, bs, q, scale);
    uwc_count_launch();
  }
  return uwc_launch_status();
}

extern "C" int uwc_swiglu(const int32_t* acc, const float* s3, const float* sw, int m, int I, float* h, void* stream) {
  if (!acc || !s3 || !sw || !h || m < 0 || I <= 0) return UWC_ERR_ARG;
  if (m > 65535) return UWC_ERR_SHAPE;
  UWC_CHECK_DEVICE();
  if (m == 0) return UWC_OK;
  k_swiglu<<<dim3((I + 255) / 256, m), 256, 0, (cudaStream_t)stream>>>(acc, s3, sw, I, h);
  uwc_count_launch();
  return uwc_launch_status();
}

extern "C" int uwc_dequant_residual(const int32_t* acc, const float* s, const float* sw, const float* x, int m, int k,
                                    float* out, void* stream) {
  if (!acc || !s || !sw || !out || m < 0 || k <= 0 || k % 4) return UWC_ERR_ARG;
  if (!aligned16(acc) || !aligned16(sw) || (x && !aligned16(x)) || !aligned16(out)) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  const uint64_t n4 = (uint64_t)m * k / 4;
  if (n4 == 0) return UWC_OK;
  const int grid = (int)std::min<uint64_t>((n4 + 255) / 256, (uint64_t)uwc_num_sms() * 16);
  k_dequant_residual<<<grid, 256, 0, (cudaStream_t)stream>>>(acc, s, sw, x, k, n4, out);
  uwc_count_launch();
  return uwc_launch_status();
}

namespace {
int qkv_post_launch(const int32_t* acc, const float* s1, const float* sw, const float* qnw, const float* knw,
                    const float* cos_t, const float* sin_t, int N, int T, int H, int Hkv, double eps, int qknorm,
                    int8_t* qq, float* qs, int8_t* kq, float* ks, int8_t* vq, float* vs, const int* pos0,
                    void* stream, KVDest kv = KVDest{}) {
  if (!acc || !s1 || !sw || !cos_t || !sin_t || !qq || !qs) return UWC_ERR_ARG;
  if (kv.k ? (!kv.sk || !kv.v || !kv.sv || kv.maxlen <= 0 || !pos0) : (!kq || !ks || !vq || !vs)) return UWC_ERR_ARG;
  if (qknorm && (!qnw || !knw)) return UWC_ERR_ARG;
  if (N < 0 || T <= 0 || H <= 0 || Hkv <= 0) return UWC_ERR_SHAPE;
  UWC_CHECK_DEVICE();
  if (N == 0) return UWC_OK;
  k_qkv_post<<<N, kRowThreads, 0, (cudaStream_t)stream>>>(acc, s1, sw, qnw, knw, cos_t, sin_t, T, H, Hkv,
                                                          (float)(1.0 / 128), (float)eps, qknorm, qq, qs, kq, ks, vq,
                                                          vs, pos0, kv);
  uwc_count_launch();
  return uwc_launch_status();
}
}  // namespace

extern "C" int uwc_qkv_post(const int32_t* acc, const float* s1, const float* sw, const float* qnw, const float* knw,
                            const float* cos_t, const float* sin_t, int N, int T, int H, int Hkv, double eps,
                            int qknorm, int8_t* qq, float* qs, int8_t* kq, float* ks, int8_t* vq, float* vs,
                            void* stream) {
  return qkv_post_launch(acc, s1, sw, qnw, knw, cos_t, sin_t, N, T, H, Hkv, eps, qknorm, qq, qs, kq, ks, vq, vs,
                         nullptr, stream);
}

extern "C" int uwc_qkv_post_kv(const int32_t* acc, const float* s1, const float* sw, const float* qnw,
                               const float* knw, const float* cos_table, const float* sin_table, const int* pos,
                               int N, int T, int H, int Hkv, double eps, int qknorm, int8_t* qq, float* qs,
                               int8_t* kc, float* skc, int8_t* vc, float* svc, int maxlen, void* stream) {
  if (!pos || !kc) return UWC_ERR_ARG;
  return qkv_post_launch(acc, s1, sw, qnw, knw, cos_table, sin_table, N, T, H, Hkv, eps, qknorm, qq, qs, nullptr,
                         nullptr, nullptr, nullptr, pos, stream, KVDest{kc, skc, vc, svc, maxlen});
}

extern "C" int uwc_qkv_post_at(const int32_t* acc, const float* s1, const float* sw, const float* qnw,
                               const float* knw, const float* cos_table, const float* sin_table, const int* pos,
                               int N, int T, int H, int Hkv, double eps, int qknorm, int8_t* qq, float* qs,
                               int8_t* kq, float* ks, int8_t* vq, float* vs, void* stream) {
  if (!pos) return UWC_ERR_ARG;
  return qkv_post_launch(acc, s1, sw, qnw, knw, cos_table, sin_table, N, T, H, Hkv, eps, qknorm, qq, qs, kq, ks, vq,
                         vs, pos, stream);
}
