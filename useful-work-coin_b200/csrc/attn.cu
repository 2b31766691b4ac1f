// The rest of runtime/detrt's forward on sm_100a: exact integer attention, the final RMSNorm and
// the deterministic log-softmax + greedy argmax. Bit-identical to runtime/detrt/qwen3.py.
//
//   k_attention   _attention's core (qwen3.py:254-283, GPU form runtime/detgpu/kernels.py attention)
//                 from quantized q, k, v: exact int32 Q K^T, the fp32 scale chain, causal mask,
//                 det_exp, exact int64 row sum, P = e / den, P * sv quantized to 14 bits, P V
//                 as two 7-bit limbs, each an exact int32 dot, summed in int64, times the scale.
//   k_rmsnorm     det_rmsnorm (core.py:151-159) to fp32 (the final norm).
//   k_logprobs    logprobs (qwen3.py:302-312): max, det_exp, exact row sum (2^18 terms), det_log;
//                 the greedy token is the first index of the row's maximal log-probability
//                 (generate_greedy, qwen3.py:315-329).
//
// Attention layout: one CTA per (sequence, query head, block of QT query rows). The CTA keeps its
// rows' scores in shared memory (QT x S floats), overwritten in place by e, P * sv and finally the
// 14-bit integer probabilities; V is staged per 64-key tile transposed (dims x keys) so the P V
// dot products run four keys per dp4a. Keys and values are read with strides, so the same kernel
// serves the prefill layout (token-major, the detgpu call) and a KV cache (head-major, decode).
// A decode token (Tq = 1) runs k_attn_decode instead: a cluster of 8 CTAs per (sequence, KV head)
// splits the keys and combines its reductions through distributed shared memory.
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include <cooperative_groups.h>

#include "det_math.cuh"
#include "uwc_device.cuh"
#include "uwc_host.h"

namespace {

constexpr int kAttnThreads = 256;
constexpr int kHd = 128;               // head dim (the detgpu attention kernels' fixed width)
constexpr int kTileKeys = 64;          // keys per staged V tile
constexpr int kVtPitch = kTileKeys + 4;  // bytes per transposed V row (padding against bank conflicts)
constexpr int kPLevels = 16383;        // qwen3.py P_LEVELS: 14-bit probabilities
constexpr int kMaxKeysLog2 = 20;       // qwen3.py MAX_KEYS = 2^20 (exact_rowsum's length bound)

// detrt.core.det_log (core.py:130-143): x = m 2^e, log m = 2 atanh((m - 1) / (m + 1)) as the odd
// series to s^15 in Horner form; one rounding per op.
__device__ __forceinline__ float det_log(float x) {
  int e;
  float m = frexpf(x, &e);  // m in [0.5, 1)
  m = __fmul_rn(m, 2.0f);
  const float ef = (float)(e - 1);
  const float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  const float s2 = __fmul_rn(s, s);
  float acc = (float)(1.0 / 15);
  acc = __fadd_rn(__fmul_rn(acc, s2), (float)(1.0 / 13));
  acc = __fadd_rn(__fmul_rn(acc, s2), (float)(1.0 / 11));
  acc = __fadd_rn(__fmul_rn(acc, s2), (float)(1.0 / 9));
  acc = __fadd_rn(__fmul_rn(acc, s2), (float)(1.0 / 7));
  acc = __fadd_rn(__fmul_rn(acc, s2), (float)(1.0 / 5));
  acc = __fadd_rn(__fmul_rn(acc, s2), (float)(1.0 / 3));
  acc = __fadd_rn(__fmul_rn(acc, s2), 1.0f);
  const float lm = __fmul_rn(__fmul_rn(acc, s), 2.0f);
  return __fadd_rn(__fmul_rn(ef, (float)0.6931471805599453), lm);
}

// Exact fixed-point row sum term (core.py:85-108): the int64 image of v at scale 2^sh.
__device__ __forceinline__ long long fixed_term(float v, double up) { return __double2ll_rn((double)v * up); }

__device__ __forceinline__ int fixed_shift(float amax, int L) {
  int e;
  frexpf(amax, &e);
  return min(max((62 - L) - e, -1000), 1000);
}

struct AttnArgs {
  const int8_t* qq;   // (N_q, H, 128), row n = b * Tq + t
  const float* qs;    // (N_q, H)
  const int8_t* kc;   // keys: element (b, j, g, d) at b * kv_seq + j * kv_tok + g * kv_head + d
  const float* ks;    // key scales: (b, j, g) at b * s_seq + j * s_tok + g * s_head
  const int8_t* vc;   // values, same strides as the keys
  const float* vs;    // value scales, same strides as the key scales
  long long kv_seq, kv_tok, kv_head, s_seq, s_tok, s_head;
  int Tq, start, H, Hkv;
  float inv_sqrt_hd;
  float* out;         // (N_q, H * 128)
  const int* start_dev;   // when set, the start position is read here (one graph for every decode step)
};

// Row r of this CTA is query t = t0 + r at absolute position start + t; it sees keys 0..start + t.
// QT <= 8 rows; each row is owned by WPR = 8 / QT warps, which split its keys (a single decode row
// uses the whole CTA). Partial maxima and integer sums combine exactly, in any order.
template <int QT>
__global__ void __launch_bounds__(kAttnThreads) k_attention(const AttnArgs a, int spitch) {
  constexpr int NW = kAttnThreads / 32, WPR = NW / QT;
  static_assert(QT >= 1 && QT <= NW && NW % QT == 0, "rows per CTA");
  extern __shared__ __align__(16) uint8_t sm[];
  float* sc = reinterpret_cast<float*>(sm);                              // QT x spitch
  uint32_t* qrow = reinterpret_cast<uint32_t*>(sm + (size_t)QT * spitch * 4);  // QT x 32 words
  uint8_t* vt = reinterpret_cast<uint8_t*>(qrow + QT * 32);             // 128 x kVtPitch
  __shared__ float s_qs[QT], s_sp[QT], s_red[QT][WPR];
  __shared__ long long s_redl[QT][WPR];
  // rows split over several warps combine their P V partials here (after the V tile)
  long long* s_out = reinterpret_cast<long long*>(vt + kHd * kVtPitch);   // QT x WPR x 128

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = warp / WPR, part = warp % WPR;              // this warp's row and key split
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H, g = h / (a.H / a.Hkv);
  const int t0 = blockIdx.y * QT;
  const int nrows = min(QT, a.Tq - t0);
  const bool live = r < nrows;
  const int start = a.start_dev ? __ldg(a.start_dev) : a.start;
  const int S = start + t0 + nrows;                        // keys this CTA needs
  const int8_t* kb = a.kc + b * a.kv_seq + g * a.kv_head;
  const int8_t* vb = a.vc + b * a.kv_seq + g * a.kv_head;
  const float* ksb = a.ks + b * a.s_seq + g * a.s_head;
  const float* vsb = a.vs + b * a.s_seq + g * a.s_head;

  // ---- queries (int8 rows) and their scales
  for (int i = tid; i < QT * 32; i += kAttnThreads) {
    const int rr = i >> 5;
    qrow[i] = rr < nrows ? reinterpret_cast<const uint32_t*>(a.qq + ((size_t)(b * a.Tq + t0 + rr) * a.H + h) * kHd)[i & 31]
                         : 0u;
  }
  if (tid < QT) s_qs[tid] = tid < nrows ? a.qs[(size_t)(b * a.Tq + t0 + tid) * a.H + h] : 0.f;
  __syncthreads();

  // ---- scores: fmul(fmul(fmul(float(q . k), qs), ks), 1/sqrt(hd)), -inf past the query's position
  for (int j = tid; j < S; j += kAttnThreads) {
    uint32_t kw[32];
    const uint4* kp = reinterpret_cast<const uint4*>(kb + (size_t)j * a.kv_tok);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint4 v = __ldg(kp + i);
      kw[4 * i] = v.x; kw[4 * i + 1] = v.y; kw[4 * i + 2] = v.z; kw[4 * i + 3] = v.w;
    }
    const float ksj = __ldg(ksb + (size_t)j * a.s_tok);
#pragma unroll 1
    for (int rr = 0; rr < nrows; rr++) {
      const uint4* qv = reinterpret_cast<const uint4*>(qrow + rr * 32);
      int dot = 0;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint4 qw = qv[i];
        dot = __dp4a((int)kw[4 * i], (int)qw.x, dot);
        dot = __dp4a((int)kw[4 * i + 1], (int)qw.y, dot);
        dot = __dp4a((int)kw[4 * i + 2], (int)qw.z, dot);
        dot = __dp4a((int)kw[4 * i + 3], (int)qw.w, dot);
      }
      const float v = __fmul_rn(__fmul_rn(__fmul_rn((float)dot, s_qs[rr]), ksj), a.inv_sqrt_hd);
      sc[rr * spitch + j] = j <= start + t0 + rr ? v : __int_as_float(0xff800000);
    }
  }
  __syncthreads();

  // ---- per row: max, det_exp, exact sum, P * sv, 14-bit quantization. The row's WPR warps take
  // keys j = 32 * part + lane (mod 32 * WPR) and combine their partials through shared memory.
  float* row = sc + r * spitch;
  const int j0 = 32 * part + lane, js = 32 * WPR;
  auto row_max = [&](float v) -> float {
    v = warp_maxf(v);
    if (lane == 0) s_red[r][part] = v;
    __syncthreads();
    float m = s_red[r][0];
#pragma unroll
    for (int i = 1; i < WPR; i++) m = fmaxf(m, s_red[r][i]);
    __syncthreads();
    return m;
  };
  float mx = __int_as_float(0xff800000);
  if (live)
    for (int j = j0; j < S; j += js) mx = fmaxf(mx, row[j]);
  mx = row_max(mx);
  float emax = 0.f;
  if (live)
    for (int j = j0; j < S; j += js) {
      const float e = det_exp(__fsub_rn(row[j], mx));
      row[j] = e;
      emax = fmaxf(emax, e);
    }
  emax = row_max(emax);
  const int sh = fixed_shift(emax, kMaxKeysLog2);
  long long acc = 0;
  if (live) {
    if (sh <= 100) {                 // |e| 2^sh stays a normal float below 2^62: exact in fp32
      const float up = pow2f(sh);
      for (int j = j0; j < S; j += js) acc += __float2ll_rn(__fmul_rn(row[j], up));
    } else {
      const double up = pow2d(sh);
      for (int j = j0; j < S; j += js) acc += fixed_term(row[j], up);
    }
  }
  acc = warp_sumll(acc);
  if (lane == 0) s_redl[r][part] = acc;
  __syncthreads();
  acc = 0;
#pragma unroll
  for (int i = 0; i < WPR; i++) acc += s_redl[r][i];
  const float den = __double2float_rn(__ll2double_rn(acc) * pow2d(-sh));
  float pmax = 0.f;
  if (live)
    for (int j = j0; j < S; j += js) {
      const float pv = __fmul_rn(__fdiv_rn(row[j], den), __ldg(vsb + (size_t)j * a.s_tok));
      row[j] = pv;
      pmax = fmaxf(pmax, pv);
    }
  pmax = row_max(pmax);
  const float sp = __fdiv_rn(fmaxf(pmax, 1e-30f), (float)kPLevels);
  const int Sp = (S + kTileKeys - 1) / kTileKeys * kTileKeys;
  if (live)
    for (int j = j0; j < Sp; j += js) {
      int pi = 0;
      if (j < S) pi = int_of_small(fminf(fmaxf(rint_small(__fdiv_rn(row[j], sp)), 0.f), (float)kPLevels));
      reinterpret_cast<int*>(row)[j] = pi;
    }
  if (lane == 0 && part == 0) s_sp[r] = sp;
  __syncthreads();

  // ---- P V: lane l owns dims l, l + 32, l + 64, l + 96 of its row; the row's warps split each
  // 64-key tile's 4-key groups. V is staged per tile transposed (vt[dim][key], 4 keys a word), so
  // each dp4a adds four keys' hi (resp. lo) limbs times their values: exact int32 partial sums
  // (|sum| < 127 * 127 * S), combined as (hi << 7) + lo in int64 (detrt sums per 1024-key chunk).
  int acc_hi[4] = {0, 0, 0, 0}, acc_lo[4] = {0, 0, 0, 0};
  const uint32_t* vtw = reinterpret_cast<const uint32_t*>(vt);
  for (int jt = 0; jt < S; jt += kTileKeys) {
    for (int bi = tid; bi < (kTileKeys / 4) * (kHd / 4); bi += kAttnThreads) {
      const int kg = bi >> 5, dg = bi & 31;
      uint32_t w[4];
#pragma unroll
      for (int x = 0; x < 4; x++) {
        const int j = jt + 4 * kg + x;
        w[x] = j < S ? __ldg(reinterpret_cast<const uint32_t*>(vb + (size_t)j * a.kv_tok) + dg) : 0u;
      }
      const uint32_t lo01 = __byte_perm(w[0], w[1], 0x5140), hi01 = __byte_perm(w[0], w[1], 0x7362);
      const uint32_t lo23 = __byte_perm(w[2], w[3], 0x5140), hi23 = __byte_perm(w[2], w[3], 0x7362);
      uint32_t* dst = reinterpret_cast<uint32_t*>(vt + (size_t)(4 * dg) * kVtPitch) + kg;
      dst[0] = __byte_perm(lo01, lo23, 0x5410);
      dst[kVtPitch / 4] = __byte_perm(lo01, lo23, 0x7632);
      dst[2 * kVtPitch / 4] = __byte_perm(hi01, hi23, 0x5410);
      dst[3 * kVtPitch / 4] = __byte_perm(hi01, hi23, 0x7632);
    }
    __syncthreads();
    if (live) {
      const int4* prow = reinterpret_cast<const int4*>(sc + r * spitch + jt);
#pragma unroll 4
      for (int kg = part; kg < kTileKeys / 4; kg += WPR) {
        const int4 p4 = prow[kg];
        // 14-bit probabilities -> four 7-bit hi limbs and four 7-bit lo limbs, one byte each
        const uint32_t lo4 =
            __byte_perm(__byte_perm(p4.x, p4.y, 0x0040), __byte_perm(p4.z, p4.w, 0x0040), 0x5410) & 0x7F7F7F7Fu;
        const uint32_t hi4 = __byte_perm(__byte_perm(p4.x << 1, p4.y << 1, 0x0051),
                                         __byte_perm(p4.z << 1, p4.w << 1, 0x0051), 0x5410);
#pragma unroll
        for (int y = 0; y < 4; y++) {
          const int vv = (int)vtw[(lane + 32 * y) * (kVtPitch / 4) + kg];
          acc_hi[y] = __dp4a((int)hi4, vv, acc_hi[y]);
          acc_lo[y] = __dp4a((int)lo4, vv, acc_lo[y]);
        }
      }
    }
    __syncthreads();
  }
  // o = fmul(float(acc), sp), acc the exact int64 sum over the row's warps (qwen3.py:276-282)
  float* o = a.out + (size_t)(b * a.Tq + t0 + r) * a.H * kHd + h * kHd;
  if constexpr (WPR == 1) {
    if (live)
#pragma unroll
      for (int y = 0; y < 4; y++) o[lane + 32 * y] = __fmul_rn(__ll2float_rn(((long long)acc_hi[y] << 7) + acc_lo[y]), s_sp[r]);
  } else {
  #pragma unroll
    for (int y = 0; y < 4; y++) s_out[(r * WPR + part) * kHd + lane + 32 * y] = ((long long)acc_hi[y] << 7) + acc_lo[y];
    __syncthreads();
    if (live && part == 0) {
  #pragma unroll
      for (int y = 0; y < 4; y++) {
        long long t = 0;
  #pragma unroll
        for (int i = 0; i < WPR; i++) t += s_out[(r * WPR + i) * kHd + lane + 32 * y];
        o[lane + 32 * y] = __fmul_rn(__ll2float_rn(t), s_sp[r]);
      }
    }
  }
}

// ---- decode: one query token per sequence (Tq = 1), the keys split over a cluster of CTAs.
// A cluster of CL (4, or kDecCluster for long caches) CTAs serves one (sequence, KV head) pair and
// all HPG = H / Hkv query heads that read it, so each key and value row is loaded once per token. CTA `rank` owns keys
// [rank S / C, (rank + 1) S / C). The softmax's four row reductions (max, max of e, the exact int64
// sum, max of P * sv) and the int64 P V partials combine across the cluster through distributed
// shared memory: max and integer addition are exact in any order, so the result is bit-identical
// to the single-CTA kernel and to detrt.
constexpr int kDecCluster = 8;

// the four reductions' exchange slots (one per reduction, so no slot is rewritten) and the partials
template <int HPG>
struct DecShared {
  float red[3][8];         // per-warp partials of the three maxima (one slot set each: no reuse)
  long long redl[2][8];    // per-warp partials of the row sum (and of its rare second pass)
  float xf[3][HPG];        // row max, max of e, max of P * sv: this CTA's values
  long long xl[2][HPG];    // exact row sum at the presumed shift (and at the true one): this CTA's value
  float sp[HPG];
  long long part[HPG][kHd];  // this CTA's P V partial, read by the cluster's final reduction
};

// Global -> shared copies that bypass registers (cp.async), issued in commit groups; a thread
// waits for its own groups, a barrier then publishes them to the CTA.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int HPG, int CL>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(kAttnThreads)
    k_attn_decode(const AttnArgs a, int lpitch) {
  constexpr int NW = kAttnThreads / 32, WPR = NW / HPG;
  static_assert(HPG >= 1 && HPG <= NW && NW % HPG == 0, "query heads per KV head");
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t sm[];
  uint32_t* vrows = reinterpret_cast<uint32_t*>(sm);                               // lpitch x 32 words
  float* sc = reinterpret_cast<float*>(sm + (size_t)lpitch * kHd);                 // HPG x lpitch
  float* svs = sc + (size_t)HPG * lpitch;                                          // lpitch value scales
  uint32_t* qrow = reinterpret_cast<uint32_t*>(svs + lpitch);                      // HPG x 32 words
  long long* s_out = reinterpret_cast<long long*>(qrow + HPG * 32);                // NW x 128
  __shared__ DecShared<HPG> ds;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = warp / WPR, part = warp % WPR;
  const int rank = (int)cluster.block_rank();
  const int pair = blockIdx.x / CL;
  const int b = pair / a.Hkv, g = pair % a.Hkv;
  const int start = a.start_dev ? __ldg(a.start_dev) : a.start;
  const int S = start + 1;
  const int k0 = (int)((long long)rank * S / CL), k1 = (int)((long long)(rank + 1) * S / CL);
  const int nk = k1 - k0;
  const int8_t* kb = a.kc + b * a.kv_seq + g * a.kv_head;
  const int8_t* vb = a.vc + b * a.kv_seq + g * a.kv_head;
  const float* ksb = a.ks + b * a.s_seq + g * a.s_head;
  const float* vsb = a.vs + b * a.s_seq + g * a.s_head;
  const int h0 = g * HPG;

  // Loads in the order they are needed: the thread's first key row (registers), then by cp.async
  // the query rows (group 1), the value scales (group 2) and the value rows (group 3), which
  // stream into shared memory while the scores and the softmax run.
  uint32_t kw[32];
  float ksj = 0.f;
  auto load_key = [&](int jl) {
    const uint4* kp = reinterpret_cast<const uint4*>(kb + (size_t)(k0 + jl) * a.kv_tok);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint4 v = __ldg(kp + i);
      kw[4 * i] = v.x; kw[4 * i + 1] = v.y; kw[4 * i + 2] = v.z; kw[4 * i + 3] = v.w;
    }
    ksj = __ldg(ksb + (size_t)(k0 + jl) * a.s_tok);
  };
  if (tid < nk) load_key(tid);
  for (int i = tid; i < HPG * 8; i += kAttnThreads)
    cp_async16(qrow + 4 * i, a.qq + ((size_t)b * a.H + h0 + (i >> 3)) * kHd + (i & 7) * 16);
  cp_async_commit();
  for (int j = tid; j < nk; j += kAttnThreads) cp_async4(svs + j, vsb + (size_t)(k0 + j) * a.s_tok);
  cp_async_commit();
  for (int i = tid; i < nk * 8; i += kAttnThreads)
    cp_async16(vrows + (size_t)(i >> 3) * 32 + (i & 7) * 4, vb + (size_t)(k0 + (i >> 3)) * a.kv_tok + (i & 7) * 16);
  cp_async_commit();
  cp_async_wait<2>();   // the query rows
  __syncthreads();

  // ---- scores of this CTA's keys for every query head of the group
  for (int jl = tid; jl < nk; jl += kAttnThreads) {
    if (jl != tid) load_key(jl);
#pragma unroll
    for (int rr = 0; rr < HPG; rr++) {
      const uint4* qv = reinterpret_cast<const uint4*>(qrow + rr * 32);
      int dot = 0;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint4 qw = qv[i];
        dot = __dp4a((int)kw[4 * i], (int)qw.x, dot);
        dot = __dp4a((int)kw[4 * i + 1], (int)qw.y, dot);
        dot = __dp4a((int)kw[4 * i + 2], (int)qw.z, dot);
        dot = __dp4a((int)kw[4 * i + 3], (int)qw.w, dot);
      }
      const float qsr = __ldg(a.qs + (size_t)b * a.H + h0 + rr);
      sc[rr * lpitch + jl] = __fmul_rn(__fmul_rn(__fmul_rn((float)dot, qsr), ksj), a.inv_sqrt_hd);
    }
  }
  __syncthreads();

  // row reduction over this CTA (the row's WPR warps), then over the cluster
  float* row = sc + r * lpitch;
  const int j0 = 32 * part + lane, js = 32 * WPR;
  auto cta_max = [&](float v, int slot) -> float {
    v = warp_maxf(v);
    if (lane == 0) ds.red[slot][warp] = v;
    __syncthreads();
    float m = ds.red[slot][r * WPR];
#pragma unroll
    for (int i = 1; i < WPR; i++) m = fmaxf(m, ds.red[slot][r * WPR + i]);
    return m;
  };
  auto cluster_max = [&](float v, int slot) -> float {
    v = cta_max(v, slot);
    if (part == 0 && lane == 0) ds.xf[slot][r] = v;
    cluster.sync();
#pragma unroll
    for (int q = 0; q < CL; q++) v = fmaxf(v, cluster.map_shared_rank(&ds.xf[slot][r], q)[0]);
    return v;
  };
  // this CTA's exact fixed-point sum of the row's e at shift sh, into exchange slot `slot`
  auto cta_sum = [&](int sh, int slot) {
    long long acc = 0;
    if (sh <= 100) {                 // |e| 2^sh stays a normal float below 2^62: exact in fp32
      const float up = pow2f(sh);
      for (int j = j0; j < nk; j += js) acc += __float2ll_rn(__fmul_rn(row[j], up));
    } else {
      const double up = pow2d(sh);
      for (int j = j0; j < nk; j += js) acc += fixed_term(row[j], up);
    }
    acc = warp_sumll(acc);
    if (lane == 0) ds.redl[slot][warp] = acc;
    __syncthreads();
    if (part == 0 && lane == 0) {
      long long t = 0;
#pragma unroll
      for (int i = 0; i < WPR; i++) t += ds.redl[slot][r * WPR + i];
      ds.xl[slot][r] = t;
    }
  };
  float mx = __int_as_float(0xff800000);
  for (int j = j0; j < nk; j += js) mx = fmaxf(mx, row[j]);
  mx = cluster_max(mx, 0);
  float emax = 0.f;
  for (int j = j0; j < nk; j += js) {
    const float e = det_exp(__fsub_rn(row[j], mx));
    row[j] = e;
    emax = fmaxf(emax, e);
  }
  // The sum's shift follows from the row's max of e, which is det_exp(0) = 1 (the max score's own
  // term) unless another term rounds to 2 or more: the sum at that presumed shift travels with the
  // max of e in one exchange, and only a different true shift (uniform over the cluster) costs a
  // second exchange. Either way the sum is the one at the true shift.
  const int sh_guess = fixed_shift(1.0f, kMaxKeysLog2);
  emax = cta_max(emax, 1);
  if (part == 0 && lane == 0) ds.xf[1][r] = emax;
  cta_sum(sh_guess, 0);
  cp_async_wait<1>();   // the value scales, read after this exchange
  cluster.sync();
#pragma unroll
  for (int q = 0; q < CL; q++) emax = fmaxf(emax, cluster.map_shared_rank(&ds.xf[1][r], q)[0]);
  const int sh = fixed_shift(emax, kMaxKeysLog2);
  long long acc = 0;
  if (__syncthreads_or(sh != sh_guess)) {
    cta_sum(sh, 1);
    cluster.sync();
#pragma unroll
    for (int q = 0; q < CL; q++) acc += cluster.map_shared_rank(&ds.xl[1][r], q)[0];
  } else {
#pragma unroll
    for (int q = 0; q < CL; q++) acc += cluster.map_shared_rank(&ds.xl[0][r], q)[0];
  }
  const float den = __double2float_rn(__ll2double_rn(acc) * pow2d(-sh));
  float pmax = 0.f;
  for (int j = j0; j < nk; j += js) {
    const float pv = __fmul_rn(__fdiv_rn(row[j], den), svs[j]);
    row[j] = pv;
    pmax = fmaxf(pmax, pv);
  }
  pmax = cluster_max(pmax, 2);
  const float sp = __fdiv_rn(fmaxf(pmax, 1e-30f), (float)kPLevels);
  const int nk4 = (nk + 3) & ~3;
  for (int j = j0; j < nk4; j += js) {
    int pi = 0;
    if (j < nk) pi = int_of_small(fminf(fmaxf(rint_small(__fdiv_rn(row[j], sp)), 0.f), (float)kPLevels));
    reinterpret_cast<int*>(row)[j] = pi;
  }
  if (lane == 0 && part == 0) ds.sp[r] = sp;
  cp_async_wait<0>();   // the value rows
  __syncthreads();

  // ---- P V over this CTA's keys, straight from the staged value rows: lane l owns dims 4l..4l+3;
  // four keys' words are transposed in registers so each dp4a adds four keys' hi (resp. lo) limbs
  // times one dim's values: exact int32 partial sums (|sum| < 127 * 127 * S), combined as
  // (hi << 7) + lo in int64.
  int acc_hi[4] = {0, 0, 0, 0}, acc_lo[4] = {0, 0, 0, 0};
  const int4* prow = reinterpret_cast<const int4*>(row);
#pragma unroll 4
  for (int kg = part; kg < nk4 / 4; kg += WPR) {
    const int4 p4 = prow[kg];
    const uint32_t lo4 =
        __byte_perm(__byte_perm(p4.x, p4.y, 0x0040), __byte_perm(p4.z, p4.w, 0x0040), 0x5410) & 0x7F7F7F7Fu;
    const uint32_t hi4 = __byte_perm(__byte_perm(p4.x << 1, p4.y << 1, 0x0051),
                                     __byte_perm(p4.z << 1, p4.w << 1, 0x0051), 0x5410);
    const uint32_t* vr = vrows + (size_t)(4 * kg) * 32 + lane;
    const uint32_t w0 = vr[0], w1 = vr[32], w2 = vr[64], w3 = vr[96];
    const uint32_t lo01 = __byte_perm(w0, w1, 0x5140), hi01 = __byte_perm(w0, w1, 0x7362);
    const uint32_t lo23 = __byte_perm(w2, w3, 0x5140), hi23 = __byte_perm(w2, w3, 0x7362);
    const uint32_t d4[4] = {__byte_perm(lo01, lo23, 0x5410), __byte_perm(lo01, lo23, 0x7632),
                            __byte_perm(hi01, hi23, 0x5410), __byte_perm(hi01, hi23, 0x7632)};
#pragma unroll
    for (int y = 0; y < 4; y++) {
      acc_hi[y] = __dp4a((int)hi4, (int)d4[y], acc_hi[y]);
      acc_lo[y] = __dp4a((int)lo4, (int)d4[y], acc_lo[y]);
    }
  }
#pragma unroll
  for (int y = 0; y < 4; y++) s_out[warp * kHd + 4 * lane + y] = ((long long)acc_hi[y] << 7) + acc_lo[y];
  __syncthreads();
  for (int i = tid; i < HPG * kHd; i += kAttnThreads) {
    const int rr = i / kHd, d = i % kHd;
    long long t = 0;
#pragma unroll
    for (int w = 0; w < WPR; w++) t += s_out[(rr * WPR + w) * kHd + d];
    ds.part[rr][d] = t;
  }
  cluster.sync();
  // the cluster's CTAs split the HPG x 128 outputs; each sums its share over the cluster
  for (int i = rank * kAttnThreads + tid; i < HPG * kHd; i += CL * kAttnThreads) {
    const int rr = i / kHd, d = i % kHd;
    long long t = 0;
#pragma unroll
    for (int q = 0; q < CL; q++) t += cluster.map_shared_rank(&ds.part[rr][d], q)[0];
    a.out[((size_t)b * a.H + h0 + rr) * kHd + d] = __fmul_rn(__ll2float_rn(t), ds.sp[rr]);
  }
  cluster.sync();   // no CTA leaves while another may still read its shared memory
}

// value rows, scores, value scales, query rows, per-warp P V partials
size_t dec_smem(int HPG, int lpitch) {
  return (size_t)lpitch * kHd + (size_t)HPG * lpitch * 4 + (size_t)lpitch * 4 + (size_t)HPG * 128 +
         (size_t)(kAttnThreads / 32) * kHd * 8;
}

// det_rmsnorm (core.py:151-159) of one row per CTA, float32 out.
template <int NT>
__global__ void __launch_bounds__(NT) k_rmsnorm(const float* __restrict__ x, const float* __restrict__ w, int k,
                                                float inv_d, float eps, int L, float* __restrict__ out) {
  __shared__ float red[NT / 32];
  __shared__ long long redl[NT / 32];
  const float* xr = x + (size_t)blockIdx.x * k;
  float mx = 0.f;
  for (int i = threadIdx.x; i < k; i += NT) mx = fmaxf(mx, __fmul_rn(xr[i], xr[i]));
  mx = block_maxf<NT>(mx, red);
  const int sh = fixed_shift(mx, L);
  const double up = pow2d(sh);
  long long acc = 0;
  for (int i = threadIdx.x; i < k; i += NT) acc += fixed_term(__fmul_rn(xr[i], xr[i]), up);
  acc = block_sumll<NT>(acc, redl);
  const float ss = __double2float_rn(__ll2double_rn(acc) * pow2d(-sh));
  const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, inv_d), eps)));
  float* o = out + (size_t)blockIdx.x * k;
  for (int i = threadIdx.x; i < k; i += NT) o[i] = __fmul_rn(__fmul_rn(xr[i], rr), w[i]);
}

// Larger log-probability wins; equal values keep the lower index (torch.argmax's first maximum).
__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

// logprobs of one row of logits per CTA (qwen3.py:302-312): z = lg - max, lp = z - det_log(den),
// den = exact_rowsum(det_exp(z), 2^18); optionally the first index of the maximal lp.
template <int NT>
__global__ void __launch_bounds__(NT) k_logprobs(const float* __restrict__ lg, int V, float* __restrict__ lp,
                                                 long long* __restrict__ tok) {
  __shared__ float red[NT / 32];
  __shared__ long long redl[NT / 32];
  __shared__ float rv[NT / 32];
  __shared__ int ri[NT / 32];
  const float* x = lg + (size_t)blockIdx.x * V;
  float mx = __int_as_float(0xff800000);
  for (int i = threadIdx.x; i < V; i += NT) mx = fmaxf(mx, x[i]);
  mx = block_maxf<NT>(mx, red);
  float emax = 0.f;
  for (int i = threadIdx.x; i < V; i += NT) emax = fmaxf(emax, det_exp(__fsub_rn(x[i], mx)));
  emax = block_maxf<NT>(emax, red);
  const int sh = fixed_shift(emax, 18);
  const double up = pow2d(sh);
  long long acc = 0;
  for (int i = threadIdx.x; i < V; i += NT) acc += fixed_term(det_exp(__fsub_rn(x[i], mx)), up);
  acc = block_sumll<NT>(acc, redl);
  const float lden = det_log(__double2float_rn(__ll2double_rn(acc) * pow2d(-sh)));
  float bv = __int_as_float(0xff800000);
  int bi = 0x7fffffff;
  float* o = lp ? lp + (size_t)blockIdx.x * V : nullptr;
  for (int i = threadIdx.x; i < V; i += NT) {
    const float v = __fsub_rn(__fsub_rn(x[i], mx), lden);
    if (o) o[i] = v;
    better(bv, bi, v, i);
  }
  if (!tok) return;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, bv, off);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, off);
    better(bv, bi, v2, i2);
  }
  if ((threadIdx.x & 31) == 0) {
    rv[threadIdx.x >> 5] = bv;
    ri[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int wdx = 1; wdx < NT / 32; wdx++) better(bv, bi, rv[wdx], ri[wdx]);
    tok[blockIdx.x] = bi;
  }
}

// Few rows (a decode step's greedy tokens): k_logprobs with each row split over a cluster of
// kLpCluster CTAs, CTA c owning elements [c V / C, (c + 1) V / C). The row max, the max of det_exp,
// the exact fixed-point sum and the first maximal index are combined through distributed shared
// memory; each is exact and order-free, so the outputs are k_logprobs' bits.
constexpr int kLpCluster = 8, kLpThreads = 256;   // 8: the portable cluster size
__global__ void __cluster_dims__(kLpCluster, 1, 1) __launch_bounds__(kLpThreads)
    k_logprobs_cl(const float* __restrict__ lg, int V, float* __restrict__ lp, long long* __restrict__ tok) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  __shared__ float red[kLpThreads / 32];
  __shared__ long long redl[kLpThreads / 32];
  __shared__ float rv[kLpThreads / 32];
  __shared__ int ri[kLpThreads / 32];
  __shared__ float pub_f[2];
  __shared__ long long pub_l;
  __shared__ float pub_v;
  __shared__ int pub_i;
  const int c = (int)cl.block_rank(), row = blockIdx.x / kLpCluster;
  const int i0 = (int)((long long)c * V / kLpCluster), i1 = (int)((long long)(c + 1) * V / kLpCluster);
  const float* x = lg + (size_t)row * V;
  float mx = __int_as_float(0xff800000);
  for (int i = i0 + threadIdx.x; i < i1; i += kLpThreads) mx = fmaxf(mx, x[i]);
  mx = block_maxf<kLpThreads>(mx, red);
  if (threadIdx.x == 0) pub_f[0] = mx;
  cl.sync();
  for (int q = 0; q < kLpCluster; q++) mx = fmaxf(mx, *cl.map_shared_rank(&pub_f[0], q));
  float emax = 0.f;
  for (int i = i0 + threadIdx.x; i < i1; i += kLpThreads) emax = fmaxf(emax, det_exp(__fsub_rn(x[i], mx)));
  emax = block_maxf<kLpThreads>(emax, red);
  if (threadIdx.x == 0) pub_f[1] = emax;
  cl.sync();
  for (int q = 0; q < kLpCluster; q++) emax = fmaxf(emax, *cl.map_shared_rank(&pub_f[1], q));
  const int sh = fixed_shift(emax, 18);
  const double up = pow2d(sh);
  long long acc = 0;
  for (int i = i0 + threadIdx.x; i < i1; i += kLpThreads) acc += fixed_term(det_exp(__fsub_rn(x[i], mx)), up);
  acc = block_sumll<kLpThreads>(acc, redl);
  if (threadIdx.x == 0) pub_l = acc;
  cl.sync();
  long long tot = 0;
  for (int q = 0; q < kLpCluster; q++) tot += *cl.map_shared_rank(&pub_l, q);
  const float lden = det_log(__double2float_rn(__ll2double_rn(tot) * pow2d(-sh)));
  float bv = __int_as_float(0xff800000);
  int bi = 0x7fffffff;
  float* o = lp ? lp + (size_t)row * V : nullptr;
  for (int i = i0 + threadIdx.x; i < i1; i += kLpThreads) {
    const float v = __fsub_rn(__fsub_rn(x[i], mx), lden);
    if (o) o[i] = v;
    better(bv, bi, v, i);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, bv, off);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, off);
    better(bv, bi, v2, i2);
  }
  if ((threadIdx.x & 31) == 0) {
    rv[threadIdx.x >> 5] = bv;
    ri[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kLpThreads / 32; w++) better(bv, bi, rv[w], ri[w]);
    pub_v = bv;
    pub_i = bi;
  }
  cl.sync();
  if (tok && c == 0 && threadIdx.x == 0) {
    for (int q = 1; q < kLpCluster; q++) better(bv, bi, *cl.map_shared_rank(&pub_v, q), *cl.map_shared_rank(&pub_i, q));
    tok[row] = bi;
  }
  cl.sync();   // peers keep their shared memory until rank 0 has read it
}

constexpr int kAttnSmemMax = 200 * 1024;

// scores (QT x spitch floats), query rows, the transposed V tile, and for rows split over several
// warps (QT < 8) their int64 P V partials (8 warps x 128 dims)
size_t attn_smem(int QT, int spitch) {
  return (size_t)QT * spitch * 4 + (size_t)QT * 128 + (size_t)kHd * kVtPitch + (QT < 8 ? (size_t)8 * kHd * 8 : 0);
}

// Opt in to more than 48 KiB of dynamic shared memory, once per kernel and device.
int smem_optin(const void* kernel, int bytes) {
  if (bytes <= 48 * 1024) return UWC_OK;
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({dev, kernel})) return UWC_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmemMax) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  done.insert({dev, kernel});
  return UWC_OK;
}

template <int QT>
int launch_attn(const AttnArgs& a, int B, int spitch, cudaStream_t st) {
  const int smem = (int)attn_smem(QT, spitch);
  const int rc = smem_optin((const void*)k_attention<QT>, smem + 1024);   // + its static reduction slots
  if (rc != UWC_OK) return rc;
  k_attention<QT><<<dim3(B * a.H, (a.Tq + QT - 1) / QT), kAttnThreads, smem, st>>>(a, spitch);
  uwc_count_launch();
  return uwc_launch_status();
}

template <int HPG, int CL>
int launch_decode(const AttnArgs& a, int B, int lpitch, cudaStream_t st) {
  const int smem = (int)dec_smem(HPG, lpitch);
  // the opt-in covers the static reduction slots too (their sum passes 48 KiB before the dynamic part does)
  const int rc = smem_optin((const void*)k_attn_decode<HPG, CL>, smem + (int)sizeof(DecShared<HPG>));
  if (rc != UWC_OK) return rc;
  k_attn_decode<HPG, CL><<<B * a.Hkv * CL, kAttnThreads, smem, st>>>(a, lpitch);
  uwc_count_launch();
  return uwc_launch_status();
}

}  // namespace

namespace {
int attention_impl(const int8_t* qq, const float* qs, const int8_t* kc, const float* ks, const int8_t* vc,
                   const float* vs, int B, int Tq, int start, const int* start_dev, int H, int Hkv, long long kv_seq,
                   long long kv_tok, long long kv_head, long long s_seq, long long s_tok, long long s_head,
                   float inv_sqrt_hd, float* out, void* stream) {
  if (!qq || !qs || !kc || !ks || !vc || !vs || !out) return UWC_ERR_ARG;
  if (B < 0 || Tq < 0 || start < 0 || H <= 0 || Hkv <= 0 || H % Hkv) return UWC_ERR_SHAPE;
  if ((((uintptr_t)qq) | ((uintptr_t)kc) | ((uintptr_t)vc)) & 15) return UWC_ERR_ALIGN;
  if (kv_tok % 16 || kv_head % 16 || kv_seq % 16) return UWC_ERR_ALIGN;   // 16-byte key / value rows
  UWC_CHECK_DEVICE();
  if (B == 0 || Tq == 0) return UWC_OK;
  if ((long long)B * H > 0x7fffffffLL) return UWC_ERR_SHAPE;
  const int S = start + Tq;
  const int spitch = (S + kTileKeys - 1) / kTileKeys * kTileKeys;
  AttnArgs a{qq, qs, kc, ks, vc, vs, kv_seq, kv_tok, kv_head, s_seq, s_tok, s_head, Tq, start, H, Hkv, inv_sqrt_hd,
             out, start_dev};
  cudaStream_t st = (cudaStream_t)stream;
  if (Tq == 1 && (long long)B * Hkv * kDecCluster <= 0x7fffffffLL) {
    // decode: the keys split over a cluster, all query heads of a KV head in one cluster; 4 CTAs
    // (fewer, longer chains: 16.0 vs 18.5 us at batch 8 x 2100 positions) while a CTA's share of the
    // keys fits in shared memory, else 8
    const int hpg = H / Hkv;
    for (int cl = kDecCluster / 2; cl <= kDecCluster; cl *= 2) {
      const int per = (S + cl - 1) / cl;
      const int lpitch = (per + kTileKeys - 1) / kTileKeys * kTileKeys;
      if (dec_smem(hpg, lpitch) > (size_t)kAttnSmemMax) continue;
      const bool four = cl < kDecCluster;
      switch (hpg) {
        case 1: return four ? launch_decode<1, 4>(a, B, lpitch, st) : launch_decode<1, 8>(a, B, lpitch, st);
        case 2: return four ? launch_decode<2, 4>(a, B, lpitch, st) : launch_decode<2, 8>(a, B, lpitch, st);
        case 4: return four ? launch_decode<4, 4>(a, B, lpitch, st) : launch_decode<4, 8>(a, B, lpitch, st);
        case 8: return four ? launch_decode<8, 4>(a, B, lpitch, st) : launch_decode<8, 8>(a, B, lpitch, st);
        default: break;
      }
      break;
    }
  }
  // the widest query block whose score rows fit in shared memory (and not wider than Tq needs)
  const int want = Tq >= 8 ? 8 : Tq >= 4 ? 4 : Tq >= 2 ? 2 : 1;
  for (int QT = want; QT >= 1; QT >>= 1) {
    if (attn_smem(QT, spitch) > (size_t)kAttnSmemMax) continue;
    switch (QT) {
      case 8: return launch_attn<8>(a, B, spitch, st);
      case 4: return launch_attn<4>(a, B, spitch, st);
      case 2: return launch_attn<2>(a, B, spitch, st);
      default: return launch_attn<1>(a, B, spitch, st);
    }
  }
  return UWC_ERR_SHAPE;   // more keys than one score row of shared memory holds
}

// KV cache append: token t of sequence b (token-major kq / vq rows, N = B * T) -> cache position
// pos + t, pos read from device memory. One warp per (b, t, kv head).
__global__ void __launch_bounds__(256) k_kv_append(const int8_t* __restrict__ kq, const float* __restrict__ ks,
                                                   const int8_t* __restrict__ vq, const float* __restrict__ vs, int B,
                                                   int T, int Hkv, int maxlen, const int* __restrict__ pos,
                                                   int8_t* __restrict__ kc, float* __restrict__ skc,
                                                   int8_t* __restrict__ vc, float* __restrict__ svc) {
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)B * T * Hkv) return;
  const int g = (int)(w % Hkv), n = (int)(w / Hkv), b = n / T, t = n % T;
  const int p = __ldg(pos) + t;
  if (p >= maxlen) return;
  const long long dst = ((long long)b * Hkv + g) * maxlen + p;      // (b, g, p) of the cache
  if (lane < 8)
    reinterpret_cast<uint4*>(kc + dst * kHd)[lane] = reinterpret_cast<const uint4*>(kq + w * kHd)[lane];
  else if (lane < 16)
    reinterpret_cast<uint4*>(vc + dst * kHd)[lane - 8] = reinterpret_cast<const uint4*>(vq + w * kHd)[lane - 8];
  else if (lane == 16)
    skc[dst] = ks[w];
  else if (lane == 17)
    svc[dst] = vs[w];
}
}  // namespace

// ------------------------------------------------------------------ prefill on the tensor cores
// The same attention for many query rows as three passes around two exact int8 GEMMs on tcgen05
// (uwc_gemm_batched): S = Q K^T in int32 (causal blocks only), then per query row the fp32 scale
// chain and the softmax -> 14-bit P as two 7-bit limbs [P_hi; P_lo], then O = [P_hi; P_lo] V in
// int32 and o = fmul(float((hi << 7) + lo), sp). The integer sums are exact, so the output is the
// same bits as k_attention. Query batch bt = b * H + h reads KV head g = h / (H / Hkv).
extern "C" int uwc_gemm_batched(const int8_t* A, const int8_t* B, int m, int n, int k, int nbatch, long long a_brows,
                                long long b_brows, int b_bdiv, int causal, int cshift, int qrows, int32_t* out,
                                void* stream);
namespace {
constexpr int kTcRowsPerCta = 4;   // query rows per softmax CTA (one warp each)

struct TcLayout {
  int nb, nkv, Tp, Sp, Sn;
  size_t qh, kh, vt, ksc, vsc, sint, pst, o32, sp, total;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

TcLayout tc_layout(int B, int Tq, int start, int H, int Hkv) {
  TcLayout L{};
  L.nb = B * H;
  L.nkv = B * Hkv;
  L.Tp = (Tq + 127) / 128 * 128;
  const int S = start + Tq;
  L.Sp = (S + 127) / 128 * 128;
  L.Sn = (S + 3) / 4 * 4;
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + bytes); return at; };
  L.qh = take((size_t)L.nb * L.Tp * kHd);
  L.kh = take((size_t)L.nkv * L.Sp * kHd);
  L.vt = take((size_t)L.nkv * kHd * L.Sp);
  L.ksc = take((size_t)L.nkv * L.Sp * 4);
  L.vsc = take((size_t)L.nkv * L.Sp * 4);
  L.sint = take((size_t)L.nb * L.Tp * L.Sn * 4);
  L.pst = take((size_t)L.nb * 2 * L.Tp * L.Sp);
  L.o32 = take((size_t)L.nb * 2 * L.Tp * kHd * 4);
  L.sp = take((size_t)L.nb * L.Tp * 4);
  L.total = o;
  return L;
}

// Query rows head-major: Qh[b * H + h][t] = q(b * Tq + t, h), 16 bytes per thread.
__global__ void k_tc_gather_q(const int8_t* __restrict__ qq, int B, int Tq, int H, int Tp, int8_t* __restrict__ qh) {
  const long long n = (long long)B * H * Tq * 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int part = (int)(i & 7);
    const long long row = i >> 3;                 // (b, h, t)
    const int t = (int)(row % Tq);
    const long long bh = row / Tq;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const uint4 v = reinterpret_cast<const uint4*>(qq + ((size_t)(b * Tq + t) * H + h) * kHd)[part];
    reinterpret_cast<uint4*>(qh + ((size_t)bh * Tp + t) * kHd)[part] = v;
  }
}

// Keys and the key / value scales per KV head: Kh[b * Hkv + g][j], KS, VS, for j < S.
__global__ void k_tc_gather_k(const int8_t* __restrict__ kc, const float* __restrict__ ks, const float* __restrict__ vs,
                              int B, int S, int Hkv, long long kv_seq, long long kv_tok, long long kv_head,
                              long long s_seq, long long s_tok, long long s_head, int Sp, int8_t* __restrict__ kh,
                              float* __restrict__ ksc, float* __restrict__ vsc) {
  const long long n = (long long)B * Hkv * S * 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int part = (int)(i & 7);
    const long long row = i >> 3;                 // (b, g, j)
    const int j = (int)(row % S);
    const long long bg = row / S;
    const int g = (int)(bg % Hkv), b = (int)(bg / Hkv);
    const uint4 v = *reinterpret_cast<const uint4*>(kc + b * kv_seq + j * kv_tok + g * kv_head + part * 16);
    reinterpret_cast<uint4*>(kh + ((size_t)bg * Sp + j) * kHd)[part] = v;
    if (part == 0) {
      ksc[(size_t)bg * Sp + j] = ks[b * s_seq + j * s_tok + g * s_head];
      vsc[(size_t)bg * Sp + j] = vs[b * s_seq + j * s_tok + g * s_head];
    }
  }
}

// Values transposed per KV head: Vt[b * Hkv + g][d][j] (keys contiguous: the P V GEMM's k axis).
// One CTA per (KV head, 64-key tile): the tile is staged in shared memory, then written per dim.
__global__ void __launch_bounds__(256) k_tc_transpose_v(const int8_t* __restrict__ vc, int B, int S, int Hkv,
                                                        long long kv_seq, long long kv_tok, long long kv_head, int Sp,
                                                        int8_t* __restrict__ vt) {
  __shared__ uint32_t tile[64][kHd / 4 + 1];
  const int bg = blockIdx.y, j0 = blockIdx.x * 64;
  const int g = bg % Hkv, b = bg / Hkv;
  for (int i = threadIdx.x; i < 64 * 32; i += 256) {
    const int jj = i >> 5, w = i & 31, j = j0 + jj;
    tile[jj][w] = j < S ? *reinterpret_cast<const uint32_t*>(vc + b * kv_seq + j * kv_tok + g * kv_head + 4 * w) : 0u;
  }
  __syncthreads();
  // thread: dim d, 4 consecutive keys -> one word of Vt
  for (int i = threadIdx.x; i < kHd * 16; i += 256) {
    const int d = i >> 4, kq = i & 15;
    uint32_t o = 0;
#pragma unroll
    for (int x = 0; x < 4; x++) o |= ((tile[4 * kq + x][d >> 2] >> (8 * (d & 3))) & 0xFFu) << (8 * x);
    if (j0 + 4 * kq < Sp) *reinterpret_cast<uint32_t*>(vt + ((size_t)bg * kHd + d) * Sp + j0 + 4 * kq) = o;
  }
}

// One warp per query row (batch bt, row t): the scale chain and softmax of k_attention on the
// int32 dots of S, the 14-bit P written as hi limbs (row t of the batch's P block) and lo limbs (row
// Tp + t), zero from key start + t + 1 up to the end of the P V GEMM's k range for t's row block.
// Each lane takes four consecutive keys per step (16-byte loads of S and the key scales). The
// exponentials and the exact sum share one pass at the shift of det_exp(0) = 1 (the row maximum's
// own term); a row whose max of e has another exponent sums again at its true shift.
__global__ void __launch_bounds__(kTcRowsPerCta * 32) k_tc_softmax(const int32_t* __restrict__ sint,
                                                                   const float* __restrict__ qs,
                                                                   const float* __restrict__ ksc,
                                                                   const float* __restrict__ vsc, int B, int Tq,
                                                                   int start, int H, int Hkv, int Tp, int Sp, int Sn,
                                                                   float inv_sqrt_hd, int8_t* __restrict__ pst,
                                                                   float* __restrict__ spo) {
  extern __shared__ __align__(16) float tc_rows[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long gr = (long long)blockIdx.x * kTcRowsPerCta + warp;   // (bt, t)
  if (gr >= (long long)B * H * Tq) return;
  const int t = (int)(gr % Tq);
  const int bt = (int)(gr / Tq);
  const int b = bt / H, h = bt % H, bg = b * Hkv + h / (H / Hkv);
  float* row = tc_rows + (size_t)warp * Sp;
  const int n = start + t + 1;                                    // keys this row sees
  const int n4 = (n + 3) & ~3;                                    // <= Sn <= Sp
  const int kcap = min(Sp, (start + (t / 128) * 128 + 128 + 127) / 128 * 128);
  const int32_t* srow = sint + ((size_t)bt * Tp + t) * Sn;
  const float* ksr = ksc + (size_t)bg * Sp;
  const float* vsr = vsc + (size_t)bg * Sp;
  const float qsr = qs[(size_t)(b * Tq + t) * H + h];
  float mx = __int_as_float(0xff800000);
  for (int j = 4 * lane; j < n4; j += 128) {
    const int4 d = __ldg(reinterpret_cast<const int4*>(srow + j));
    const float4 kk = __ldg(reinterpret_cast<const float4*>(ksr + j));
    float4 v;
    // float(dot) exactly: |dot| <= 127 * 127 * 128 < 2^22
    v.x = __fmul_rn(__fmul_rn(__fmul_rn(float_of_small(d.x), qsr), kk.x), inv_sqrt_hd);
    v.y = __fmul_rn(__fmul_rn(__fmul_rn(float_of_small(d.y), qsr), kk.y), inv_sqrt_hd);
    v.z = __fmul_rn(__fmul_rn(__fmul_rn(float_of_small(d.z), qsr), kk.z), inv_sqrt_hd);
    v.w = __fmul_rn(__fmul_rn(__fmul_rn(float_of_small(d.w), qsr), kk.w), inv_sqrt_hd);
    *reinterpret_cast<float4*>(row + j) = v;
    mx = fmaxf(mx, v.x);
    if (j + 1 < n) mx = fmaxf(mx, v.y);
    if (j + 2 < n) mx = fmaxf(mx, v.z);
    if (j + 3 < n) mx = fmaxf(mx, v.w);
  }
  mx = warp_maxf(mx);
  const int sh_guess = fixed_shift(1.0f, kMaxKeysLog2);
  const float up_guess = pow2f(sh_guess);
  float emax = 0.f;
  long long acc = 0;
  for (int j = 4 * lane; j < n4; j += 128) {
    float4 e = *reinterpret_cast<const float4*>(row + j);
    e.x = det_exp(__fsub_rn(e.x, mx));
    e.y = j + 1 < n ? det_exp(__fsub_rn(e.y, mx)) : 0.f;
    e.z = j + 2 < n ? det_exp(__fsub_rn(e.z, mx)) : 0.f;
    e.w = j + 3 < n ? det_exp(__fsub_rn(e.w, mx)) : 0.f;
    *reinterpret_cast<float4*>(row + j) = e;
    emax = fmaxf(fmaxf(emax, fmaxf(e.x, e.y)), fmaxf(e.z, e.w));
    acc += __float2ll_rn(__fmul_rn(e.x, up_guess)) + __float2ll_rn(__fmul_rn(e.y, up_guess)) +
           __float2ll_rn(__fmul_rn(e.z, up_guess)) + __float2ll_rn(__fmul_rn(e.w, up_guess));
  }
  emax = warp_maxf(emax);
  const int sh = fixed_shift(emax, kMaxKeysLog2);
  if (sh != sh_guess) {            // warp-uniform: the sum again at the true shift
    acc = 0;
    if (sh <= 100) {               // |e| 2^sh stays a normal float below 2^62: exact in fp32
      const float up = pow2f(sh);
      for (int j = lane; j < n; j += 32) acc += __float2ll_rn(__fmul_rn(row[j], up));
    } else {
      const double up = pow2d(sh);
      for (int j = lane; j < n; j += 32) acc += fixed_term(row[j], up);
    }
  }
  acc = warp_sumll(acc);
  const float den = __double2float_rn(__ll2double_rn(acc) * pow2d(-sh));
  float pmax = 0.f;
  for (int j = 4 * lane; j < n4; j += 128) {
    float4 e = *reinterpret_cast<const float4*>(row + j);
    const float4 sv = __ldg(reinterpret_cast<const float4*>(vsr + j));
    e.x = __fmul_rn(__fdiv_rn(e.x, den), sv.x);
    e.y = j + 1 < n ? __fmul_rn(__fdiv_rn(e.y, den), sv.y) : 0.f;
    e.z = j + 2 < n ? __fmul_rn(__fdiv_rn(e.z, den), sv.z) : 0.f;
    e.w = j + 3 < n ? __fmul_rn(__fdiv_rn(e.w, den), sv.w) : 0.f;
    *reinterpret_cast<float4*>(row + j) = e;
    pmax = fmaxf(fmaxf(pmax, fmaxf(e.x, e.y)), fmaxf(e.z, e.w));
  }
  pmax = warp_maxf(pmax);
  const float sp = __fdiv_rn(fmaxf(pmax, 1e-30f), (float)kPLevels);
  __syncwarp();
  // four consecutive keys per lane and step: one word of hi limbs, one of lo limbs
  int8_t* phi = pst + ((size_t)bt * 2 * Tp + t) * Sp;
  int8_t* plo = phi + (size_t)Tp * Sp;
  for (int j = 4 * lane; j < kcap; j += 128) {
    uint32_t hw = 0, lw = 0;
    if (j < n) {
      const float4 pv = *reinterpret_cast<const float4*>(row + j);
      const float pvs[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int x = 0; x < 4; x++) {
        int pi = 0;
        // pv / sp <= 16383 (1 + 2^-22): rint_small and int_of_small are exact here
        if (j + x < n) pi = int_of_small(fminf(fmaxf(rint_small(__fdiv_rn(pvs[x], sp)), 0.f), (float)kPLevels));
        hw |= (uint32_t)(pi >> 7) << (8 * x);
        lw |= (uint32_t)(pi & 127) << (8 * x);
      }
    }
    *reinterpret_cast<uint32_t*>(phi + j) = hw;
    *reinterpret_cast<uint32_t*>(plo + j) = lw;
  }
  if (lane == 0) spo[(size_t)bt * Tp + t] = sp;
}

// o(b * Tq + t, h, d) = fmul(float((hi << 7) + lo), sp), hi / lo the int32 P V rows t and Tp + t.
__global__ void k_tc_combine(const int32_t* __restrict__ o32, const float* __restrict__ spi, int B, int Tq, int H,
                             int Tp, float* __restrict__ out) {
  const long long n = (long long)B * H * Tq * (kHd / 4);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int d4 = (int)(i % (kHd / 4));
    const long long row = i / (kHd / 4);          // (bt, t)
    const int t = (int)(row % Tq);
    const long long bt = row / Tq;
    const int h = (int)(bt % H), b = (int)(bt / H);
    const int4 hi = reinterpret_cast<const int4*>(o32 + ((size_t)bt * 2 * Tp + t) * kHd)[d4];
    const int4 lo = reinterpret_cast<const int4*>(o32 + ((size_t)bt * 2 * Tp + Tp + t) * kHd)[d4];
    const float sp = spi[(size_t)bt * Tp + t];
    float4 o;
    o.x = __fmul_rn(__ll2float_rn(((long long)hi.x << 7) + lo.x), sp);
    o.y = __fmul_rn(__ll2float_rn(((long long)hi.y << 7) + lo.y), sp);
    o.z = __fmul_rn(__ll2float_rn(((long long)hi.z << 7) + lo.z), sp);
    o.w = __fmul_rn(__ll2float_rn(((long long)hi.w << 7) + lo.w), sp);
    reinterpret_cast<float4*>(out + ((size_t)(b * Tq + t) * H + h) * kHd)[d4] = o;
  }
}
}  // namespace

extern "C" uint64_t uwc_attention_tc_workspace_bytes(int B, int Tq, int start, int H, int Hkv) {
  if (B <= 0 || Tq <= 0 || start < 0 || H <= 0 || Hkv <= 0) return 0;
  return tc_layout(B, Tq, start, H, Hkv).total;
}

extern "C" int uwc_attention_tc(const int8_t* qq, const float* qs, const int8_t* kc, const float* ks, const int8_t* vc,
                                const float* vs, int B, int Tq, int start, int H, int Hkv, long long kv_seq,
                                long long kv_tok, long long kv_head, long long s_seq, long long s_tok,
                                long long s_head, float inv_sqrt_hd, float* out, void* workspace,
                                uint64_t workspace_bytes, void* stream) {
  if (!qq || !qs || !kc || !ks || !vc || !vs || !out || !workspace) return UWC_ERR_ARG;
  if (B <= 0 || Tq <= 0 || start < 0 || H <= 0 || Hkv <= 0 || H % Hkv) return UWC_ERR_SHAPE;
  if ((long long)start + Tq > 131072) return UWC_ERR_SHAPE;   // P V limb sums stay below 2^31
  if ((((uintptr_t)qq) | ((uintptr_t)kc) | ((uintptr_t)vc) | ((uintptr_t)out) | ((uintptr_t)workspace)) & 15)
    return UWC_ERR_ALIGN;
  if (kv_tok % 16 || kv_head % 16 || kv_seq % 16) return UWC_ERR_ALIGN;
  const TcLayout L = tc_layout(B, Tq, start, H, Hkv);
  if (workspace_bytes < L.total) return UWC_ERR_SCRATCH;
  const size_t smem = (size_t)kTcRowsPerCta * L.Sp * 4;
  if (smem > (size_t)kAttnSmemMax) return UWC_ERR_SHAPE;
  UWC_CHECK_DEVICE();
  int rc = smem_optin((const void*)k_tc_softmax, (int)smem);
  if (rc != UWC_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int8_t* qh = reinterpret_cast<int8_t*>(ws + L.qh);
  int8_t* kh = reinterpret_cast<int8_t*>(ws + L.kh);
  int8_t* vt = reinterpret_cast<int8_t*>(ws + L.vt);
  float* ksc = reinterpret_cast<float*>(ws + L.ksc);
  float* vsc = reinterpret_cast<float*>(ws + L.vsc);
  int32_t* sint = reinterpret_cast<int32_t*>(ws + L.sint);
  int8_t* pst = reinterpret_cast<int8_t*>(ws + L.pst);
  int32_t* o32 = reinterpret_cast<int32_t*>(ws + L.o32);
  float* spb = reinterpret_cast<float*>(ws + L.sp);
  const int S = start + Tq, grid = uwc_num_sms() * 8;
  k_tc_gather_q<<<grid, 256, 0, st>>>(qq, B, Tq, H, L.Tp, qh);
  uwc_count_launch();
  k_tc_gather_k<<<grid, 256, 0, st>>>(kc, ks, vs, B, S, Hkv, kv_seq, kv_tok, kv_head, s_seq, s_tok, s_head, L.Sp, kh,
                                      ksc, vsc);
  uwc_count_launch();
  k_tc_transpose_v<<<dim3(L.Sp / 64, L.nkv), 256, 0, st>>>(vc, B, S, Hkv, kv_seq, kv_tok, kv_head, L.Sp, vt);
  uwc_count_launch();
  if ((rc = uwc_launch_status()) != UWC_OK) return rc;
  const int hpg = H / Hkv;
  rc = uwc_gemm_batched(qh, kh, L.Tp, L.Sn, kHd, L.nb, L.Tp, L.Sp, hpg, 1, start, 0, sint, stream);
  if (rc != UWC_OK) return rc;
  const long long rows = (long long)L.nb * Tq;
  k_tc_softmax<<<(unsigned)((rows + kTcRowsPerCta - 1) / kTcRowsPerCta), kTcRowsPerCta * 32, smem, st>>>(
      sint, qs, ksc, vsc, B, Tq, start, H, Hkv, L.Tp, L.Sp, L.Sn, inv_sqrt_hd, pst, spb);
  uwc_count_launch();
  if ((rc = uwc_launch_status()) != UWC_OK) return rc;
  rc = uwc_gemm_batched(pst, vt, 2 * L.Tp, kHd, L.Sp, L.nb, 2LL * L.Tp, kHd, hpg, 2, start, L.Tp, o32, stream);
  if (rc != UWC_OK) return rc;
  k_tc_combine<<<grid, 256, 0, st>>>(o32, spb, B, Tq, H, L.Tp, out);
  uwc_count_launch();
  return uwc_launch_status();
}

extern "C" int uwc_attention(const int8_t* qq, const float* qs, const int8_t* kc, const float* ks, const int8_t* vc,
                             const float* vs, int B, int Tq, int start, int H, int Hkv, long long kv_seq,
                             long long kv_tok, long long kv_head, long long s_seq, long long s_tok, long long s_head,
                             float inv_sqrt_hd, float* out, void* stream) {
  return attention_impl(qq, qs, kc, ks, vc, vs, B, Tq, start, nullptr, H, Hkv, kv_seq, kv_tok, kv_head, s_seq, s_tok,
                        s_head, inv_sqrt_hd, out, stream);
}

extern "C" int uwc_attention_at(const int8_t* qq, const float* qs, const int8_t* kc, const float* ks, const int8_t* vc,
                                const float* vs, int B, int Tq, const int* start, int max_start, int H, int Hkv,
                                long long kv_seq, long long kv_tok, long long kv_head, long long s_seq,
                                long long s_tok, long long s_head, float inv_sqrt_hd, float* out, void* stream) {
  if (!start || max_start < 0) return UWC_ERR_ARG;
  // shared memory and the query-block width are sized for the largest start the caller allows
  return attention_impl(qq, qs, kc, ks, vc, vs, B, Tq, max_start, start, H, Hkv, kv_seq, kv_tok, kv_head, s_seq,
                        s_tok, s_head, inv_sqrt_hd, out, stream);
}

extern "C" int uwc_kv_append(const int8_t* kq, const float* ks, const int8_t* vq, const float* vs, int B, int T,
                             int Hkv, int maxlen, const int* pos, int8_t* kc, float* skc, int8_t* vc, float* svc,
                             void* stream) {
  if (!kq || !ks || !vq || !vs || !pos || !kc || !skc || !vc || !svc) return UWC_ERR_ARG;
  if (B < 0 || T < 0 || Hkv <= 0 || maxlen <= 0) return UWC_ERR_SHAPE;
  if ((((uintptr_t)kq) | ((uintptr_t)vq) | ((uintptr_t)kc) | ((uintptr_t)vc)) & 15) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  const long long warps = (long long)B * T * Hkv;
  if (warps == 0) return UWC_OK;
  k_kv_append<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(kq, ks, vq, vs, B, T, Hkv,
                                                                                       maxlen, pos, kc, skc, vc, svc);
  uwc_count_launch();
  return uwc_launch_status();
}


extern "C" int uwc_rmsnorm(const float* x, const float* w, int m, int k, double eps, float* out, void* stream) {
  if (!x || !w || !out || m < 0 || k <= 0) return UWC_ERR_ARG;
  UWC_CHECK_DEVICE();
  if (m == 0) return UWC_OK;
  int L = 1;
  while ((1 << L) < k) L++;
  // detrt rounds 1/d and eps from float64 to float32 (core.c32)
  k_rmsnorm<256><<<m, 256, 0, (cudaStream_t)stream>>>(x, w, k, (float)(1.0 / k), (float)eps, L, out);
  uwc_count_launch();
  return uwc_launch_status();
}

extern "C" int uwc_logprobs(const float* logits, int m, int V, float* lp, long long* tok, void* stream) {
  if (!logits || m < 0 || V <= 0 || (!lp && !tok)) return UWC_ERR_ARG;
  UWC_CHECK_DEVICE();
  if (m == 0) return UWC_OK;
  if (m < uwc_num_sms() && V >= 64 * kLpCluster)
    k_logprobs_cl<<<m * kLpCluster, kLpThreads, 0, (cudaStream_t)stream>>>(logits, V, lp, tok);
  else
    k_logprobs<1024><<<m, 1024, 0, (cudaStream_t)stream>>>(logits, V, lp, tok);
  uwc_count_launch();
  return uwc_launch_status();
}
