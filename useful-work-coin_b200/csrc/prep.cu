// Per-block / per-attempt preparation kernels of the NoisyGEMM path, sm_100a:
//   BLAKE3 Merkle commitment + cert-v3 salted seed   (ops.py:99-118, kernels.cu:138-244)
//   noise_uniform, noise_perm                        (ops.py:122-131, kernels.cu:246-301)
//   noise_rows (noising, projection limbs, maxabs)   (ops.py:134-142, kernels.cu:303-372)
//   proj_matrix, proj_corr (tensor-core projection)  (ops.py:145-168, kernels.cu:374-404)
// All of them are HBM- or latency-bound SIMT kernels; the dense work is in gemm_sm100.cu.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "uwc_device.cuh"
#include "uwc_host.h"

// ------------------------------------------------------------------ BLAKE3 tree
namespace {
constexpr int kChunksPerCta = 128;   // one thread per 1 KiB chunk
constexpr int kReduceGroup = 1024;   // CVs reduced by one CTA of the reduce kernel
constexpr int kPitch = 5;            // uint4 per staged 64-byte block (80 B pitch: conflict-free)

// Level-wise pairwise merge of `count` chaining values in shared memory, the odd trailing node
// carried up unchanged: this builds BLAKE3's left-balanced tree as long as the group starts at a
// multiple of a power of two >= its size. ROOT goes on the last merge when `is_root`.
__device__ void merge_cvs(uint32_t* cv, int count, const uint32_t* key, bool is_root, uint32_t one) {
  const int tid = threadIdx.x;
  while (count > 1) {
    const int pairs = count >> 1, odd = count & 1;
    uint32_t res[8];
    if (tid < pairs) {
      uint32_t msg[16];
#pragma unroll
      for (int i = 0; i < 16; i++) msg[i] = cv[2 * tid * 8 + i];
      const uint32_t fl = b3::PARENT | b3::KEYED | ((is_root && count == 2) ? b3::ROOT : 0u);
      b3::compress<true>(key, msg, 0, 64, fl, res, one);
    }
    __syncthreads();
    if (tid < pairs) {
#pragma unroll
      for (int i = 0; i < 8; i++) cv[tid * 8 + i] = res[i];
    }
    if (odd && tid == 0) {
#pragma unroll
      for (int i = 0; i < 8; i++) cv[pairs * 8 + i] = cv[(count - 1) * 8 + i];
    }
    __syncthreads();
    count = pairs + odd;
  }
}
}  // namespace

// Chaining values of 128 consecutive chunks, merged to one subtree CV per CTA.
__global__ void __launch_bounds__(kChunksPerCta) k_b3_chunks(const uint8_t* __restrict__ data, uint64_t nchunks,
                                                              const uint32_t* __restrict__ key,
                                                              uint32_t* __restrict__ cvs_out, uint32_t one) {
  __shared__ __align__(16) uint4 stage[2][kChunksPerCta * kPitch];
  __shared__ uint32_t cvs[kChunksPerCta * 8];
  const int tid = threadIdx.x;
  uint32_t k8[8];
#pragma unroll
  for (int i = 0; i < 8; i++) k8[i] = key[i];
  const uint64_t base = (uint64_t)blockIdx.x * kChunksPerCta;
  const int count = (int)min((uint64_t)kChunksPerCta, nchunks - base);
  const uint4* g = reinterpret_cast<const uint4*>(data) + base * 64;  // 64 uint4 per chunk
  auto fetch = [&](int buf, int blk) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int i = tid + kChunksPerCta * j, c = i >> 2, part = i & 3;
      if (c < count) stage[buf][c * kPitch + part] = __ldg(g + (uint64_t)c * 64 + blk * 4 + part);
    }
  };
  fetch(0, 0);
  __syncthreads();
  uint32_t cv[8];
#pragma unroll
  for (int i = 0; i < 8; i++) cv[i] = k8[i];
  for (int blk = 0; blk < 16; blk++) {
    if (blk + 1 < 16) fetch((blk + 1) & 1, blk + 1);
    if (tid < count) {
      uint32_t msg[16];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint4 w = stage[blk & 1][tid * kPitch + q];
        msg[4 * q] = w.x; msg[4 * q + 1] = w.y; msg[4 * q + 2] = w.z; msg[4 * q + 3] = w.w;
      }
      const uint32_t fl = b3::KEYED | (blk == 0 ? b3::CHUNK_START : 0u) | (blk == 15 ? b3::CHUNK_END : 0u) |
                          ((blk == 15 && nchunks == 1) ? b3::ROOT : 0u);
      b3::compress<true>(cv, msg, base + tid, 64, fl, cv, one);
    }
    __syncthreads();
  }
  if (tid < count) {
#pragma unroll
    for (int i = 0; i < 8; i++) cvs[tid * 8 + i] = cv[i];
  }
  __syncthreads();
  merge_cvs(cvs, count, k8, gridDim.x == 1 && nchunks > 1, one);
  if (tid < 8) cvs_out[(uint64_t)blockIdx.x * 8 + tid] = cvs[tid];
}

// Merge aligned groups of up to 1024 CVs. With `final` (one CTA) the result is the root; the
// salted seed seed = BLAKE3(prefix || BLAKE3_keyed(salt, root || dim || 0^28)) follows.
__global__ void __launch_bounds__(512) k_b3_reduce(const uint32_t* __restrict__ in, uint32_t count,
                                                   const uint32_t* __restrict__ key, uint32_t* __restrict__ out,
                                                   int final_level, const uint32_t* __restrict__ prefix,
                                                   const uint32_t* __restrict__ salt, uint32_t dim,
                                                   uint32_t* __restrict__ root_out, uint32_t* __restrict__ seed_out,
                                                   uint32_t one) {
  __shared__ uint32_t cvs[kReduceGroup * 8];
  const uint32_t base = blockIdx.x * kReduceGroup;
  const int cnt = (int)min((uint32_t)kReduceGroup, count - base);
  for (int i = threadIdx.x; i < cnt * 8; i += blockDim.x) cvs[i] = in[(uint64_t)base * 8 + i];
  uint32_t k8[8];
#pragma unroll
  for (int i = 0; i < 8; i++) k8[i] = key[i];
  __syncthreads();
  merge_cvs(cvs, cnt, k8, final_level != 0, one);
  if (!final_level) {
    if (threadIdx.x < 8) out[(uint64_t)blockIdx.x * 8 + threadIdx.x] = cvs[threadIdx.x];
    return;
  }
  if (threadIdx.x == 0) {
    uint32_t root[8];
#pragma unroll
    for (int i = 0; i < 8; i++) root[i] = cvs[i];
    if (root_out) {
#pragma unroll
      for (int i = 0; i < 8; i++) root_out[i] = root[i];
    }
    if (seed_out) {
      uint32_t msg[16], bound[8], s8[8], seed[8];
#pragma unroll
      for (int i = 0; i < 8; i++) { msg[i] = root[i]; msg[8 + i] = 0u; s8[i] = salt[i]; }
      msg[8] = dim;
      b3::hash64<true>(s8, msg, bound, one);
#pragma unroll
      for (int i = 0; i < 8; i++) { msg[i] = prefix[i]; msg[8 + i] = bound[i]; }
      b3::hash64<true>(nullptr, msg, seed, one);
#pragma unroll
      for (int i = 0; i < 8; i++) seed_out[i] = seed[i];
    }
  }
}

// ------------------------------------------------------------------ noise
__device__ __forceinline__ void random_hash(uint32_t index, const uint32_t* label, const uint32_t* key, int prepend,
                                            uint32_t* out) {
  uint32_t msg[16], k8[8];
#pragma unroll
  for (int i = 0; i < 8; i++) { msg[i] = 0u; msg[8 + i] = label[i]; k8[i] = key[i]; }
  msg[prepend] = 1u + index;
  b3::hash64(k8, msg, out);
}

__global__ void __launch_bounds__(256) k_noise_uniform(int8_t* __restrict__ out, uint32_t nblocks,
                                                       const uint32_t* __restrict__ label,
                                                       const uint32_t* __restrict__ key, int32_t* __restrict__ zero_me,
                                                       int zero_n, int32_t* __restrict__ zero2, int zero2_n) {
  const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
  if (zero_me && b < (uint32_t)zero_n) zero_me[b] = 0;
  if (zero2 && b < (uint32_t)zero2_n) zero2[b] = 0;
  if (b >= nblocks) return;
  uint32_t h[8], o[8];
  random_hash(b, label, key, 0, h);
#pragma unroll
  for (int i = 0; i < 8; i++) {
    // per byte (x & 63) - 32 as int8: subtracting 32 is adding 0xE0 modulo 256 in each byte lane.
    const uint32_t w = h[i] & 0x3F3F3F3Fu;
    o[i] = __vadd4(w, 0xE0E0E0E0u);
  }
  uint4* dst = reinterpret_cast<uint4*>(out + (uint64_t)b * 32);
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

__global__ void __launch_bounds__(128) k_noise_perm(uint32_t* __restrict__ out, uint32_t k, uint32_t r,
                                                    const uint32_t* __restrict__ label,
                                                    const uint32_t* __restrict__ key) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i * 8 >= k) return;
  uint32_t h[8];
  random_hash(i, label, key, 1, h);
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const uint32_t l = i * 8 + j;
    if (l < k) {
      const uint32_t first = h[j] & (r - 1);
      const uint32_t second = first ^ (1u + __umulhi(r - 1, h[j]));
      out[l] = first | (second << 16);
    }
  }
}

// ------------------------------------------------------------------ noise_rows
namespace {
constexpr int kNrRows = 8;       // row multiple of the noise_rows call (the reference's rows per CTA)
constexpr int kNaRows = 32;      // rows per staged group of the noising-only kernel
constexpr int kNaCtasPerSm = 4;  // its resident CTAs per SM (persistent grid, <= 64 registers)
}

// Noising only (no projection): dst = src + E[:, first] - E[:, second], row by row. Persistent
// CTAs (a few per SM) each take an even share of the rows, so no second partial wave leaves most
// SMs idle; the share is walked in groups of kNaRows rows whose E rows are staged in shared memory.
// Thread q owns 16 consecutive columns: their permutation pairs stay in registers for the CTA's
// whole share, A is read and ApEA written in coalesced 16-byte vectors.
// Values stay in int8 without wrapping for |src| <= 64, |E| <= 32 (kernels.cu:310-372).
__global__ void __launch_bounds__(256, kNaCtasPerSm) k_noise_add(const int8_t* __restrict__ src, int rows, int k,
                                                                 int r, const int8_t* __restrict__ E,
                                                                 const uint32_t* __restrict__ Pn,
                                                                 int8_t* __restrict__ dst, int8_t* __restrict__ corr,
                                                                 int ecopy_off, int lmax) {
  __shared__ __align__(16) int8_t Es[kNaRows * 256];
  const int r0 = (int)((int64_t)blockIdx.x * rows / gridDim.x);
  const int r1 = (int)((int64_t)(blockIdx.x + 1) * rows / gridDim.x);
  const int nq = k >> 4;
  for (int g0 = r0; g0 < r1; g0 += kNaRows) {
    const int nr = min(kNaRows, r1 - g0);
    if (g0 != r0) __syncthreads();   // the previous group's E rows are no longer read
    for (int i = threadIdx.x; i < nr * r; i += blockDim.x) Es[i] = E[(uint64_t)g0 * r + i];
    __syncthreads();
    if (corr && ecopy_off >= 0) {
      // the E half of every correction limb: [X_li | E] (kernels.cu:360-368)
      const uint64_t limb_stride = (uint64_t)rows * 2 * r;
      for (int i = threadIdx.x; i < nr * r; i += blockDim.x) {
        const int rr = i / r, j = i - rr * r;
        for (int li = 0; li < lmax; li++) corr[li * limb_stride + (uint64_t)(g0 + rr) * 2 * r + ecopy_off + j] = Es[i];
      }
    }
    for (int q = threadIdx.x; q < nq; q += blockDim.x) {
      uint32_t pf[16];
      const uint4* pn4 = reinterpret_cast<const uint4*>(Pn + 16 * q);
#pragma unroll
      for (int v = 0; v < 4; v++) {
        const uint4 p = __ldg(pn4 + v);
        pf[4 * v] = p.x; pf[4 * v + 1] = p.y; pf[4 * v + 2] = p.z; pf[4 * v + 3] = p.w;
      }
#pragma unroll 4
      for (int rr = 0; rr < nr; rr++) {
        const uint64_t off = (uint64_t)(g0 + rr) * k + 16 * q;
        const uint4 w = __ldcs(reinterpret_cast<const uint4*>(src + off));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        const int8_t* er = Es + rr * r;
        uint32_t o[4];
#pragma unroll
        for (int v = 0; v < 4; v++) {
          uint32_t ov = 0;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const uint32_t p = pf[4 * v + j];
            const int nv = (int)(int8_t)(ws[v] >> (8 * j)) + (int)er[p & 0xFFFFu] - (int)er[p >> 16];
            ov |= (uint32_t)(uint8_t)(int8_t)nv << (8 * j);
          }
          o[v] = ov;
        }
        __stcs(reinterpret_cast<uint4*>(dst + off), make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
  }
}

// One pass over rows of src (reference kernels.cu:310-372, noise_rows): any of
//   noising      dst = src + E[:, first] - E[:, second] under the permutation Pn;
//   projection   proj[row][j] = sum of src[row][l] over the columns l with first(l) == j minus the
//                sum over second(l) == j under Pp (the X / Y terms of the exact denoise), written as
//                lmax balanced base-128 limbs at corr[li][row][corr_off + j], max |proj| folded into
//                *maxabs;
//   E copy       E[row] into corr[li][row][ecopy_off + j] for every limb.
// Gather design: every CTA first inverts Pp into per-column index lists in shared memory (a counting
// sort whose positions come from shared-memory counters: the order inside a list is arbitrary and
// the integer sums do not depend on it), then walks its share of the rows: the row (and its E row)
// is staged in shared memory, the noised row is written from it, and the threads assigned to
// column j add up the bytes of j's two lists, so no value is scattered. The tensor-core path
// (k_proj_matrix + the split-K GEMM + k_proj_corr) computes the same integers; the tests compare them.
namespace {
constexpr int kPrThreads = 256;
}

__global__ void __launch_bounds__(kPrThreads)
    k_noise_project(const int8_t* __restrict__ src, int rows, int k, int r, const int8_t* __restrict__ E,
                    const uint32_t* __restrict__ Pn, int8_t* __restrict__ dst, const uint32_t* __restrict__ Pp,
                    int8_t* __restrict__ corr, int corr_off, int ecopy_off, int32_t* __restrict__ maxabs, int lmax) {
  extern __shared__ __align__(16) uint8_t pr_smem[];
  // [row k][pn k u32 (noising)][plist k u16][mlist k u16][E row 256][red 256 int][pstart r+1]
  // [mstart r+1][pcur r][mcur r]: every uint4-accessed part starts on a 16-byte boundary (k % 16 == 0)
  int8_t* const row_s = reinterpret_cast<int8_t*>(pr_smem);
  uint32_t* const pn_s = reinterpret_cast<uint32_t*>(pr_smem + k);
  uint16_t* const plist = reinterpret_cast<uint16_t*>(pr_smem + k + (dst ? 4 * k : 0));
  uint16_t* const mlist = plist + k;
  int8_t* const es = reinterpret_cast<int8_t*>(mlist + k);
  int* const red = reinterpret_cast<int*>(es + 256);
  int* const pstart = red + kPrThreads;
  int* const mstart = pstart + (r + 1);
  int* const pcur = mstart + (r + 1);
  int* const mcur = pcur + r;
  const int tid = threadIdx.x;
  const int r0 = (int)((int64_t)blockIdx.x * rows / gridDim.x);
  const int r1 = (int)((int64_t)(blockIdx.x + 1) * rows / gridDim.x);
  if (r0 >= r1) return;
  const uint64_t limb_stride = (uint64_t)rows * 2 * r;
  if (dst)
    for (int q = tid; q < (k >> 2); q += kPrThreads)
      reinterpret_cast<uint4*>(pn_s)[q] = __ldg(reinterpret_cast<const uint4*>(Pn) + q);
  if (Pp) {
    // counting sort of the k columns by first (plus lists) and by second (minus lists); pairs
    // naming a column >= r are not valid permutations and are left out of both lists
    for (int j = tid; j <= r; j += kPrThreads) pstart[j] = mstart[j] = 0;
    __syncthreads();
    for (int l = tid; l < k; l += kPrThreads) {
      const uint32_t p = __ldg(Pp + l);
      if ((p & 0xFFFFu) < (uint32_t)r) atomicAdd(&pstart[(p & 0xFFFFu) + 1], 1);
      if ((p >> 16) < (uint32_t)r) atomicAdd(&mstart[(p >> 16) + 1], 1);
    }
    __syncthreads();
    if (tid == 0) {
      for (int j = 0; j < r; j++) pstart[j + 1] += pstart[j];
    } else if (tid == 32) {
      for (int j = 0; j < r; j++) mstart[j + 1] += mstart[j];
    }
    __syncthreads();
    for (int j = tid; j < r; j += kPrThreads) {
      pcur[j] = pstart[j];
      mcur[j] = mstart[j];
    }
    __syncthreads();
    for (int l = tid; l < k; l += kPrThreads) {
      const uint32_t p = __ldg(Pp + l);
      if ((p & 0xFFFFu) < (uint32_t)r) plist[atomicAdd(&pcur[p & 0xFFFFu], 1)] = (uint16_t)l;
      if ((p >> 16) < (uint32_t)r) mlist[atomicAdd(&mcur[p >> 16], 1)] = (uint16_t)l;
    }
  }
  __syncthreads();
  const int parts = kPrThreads / r;   // threads per column: 4 (r 64), 2 (r 128), 1 (r 256)
  const int j = tid % r, part = tid / r;
  const bool want_e = E && (dst || (corr && ecopy_off >= 0));
  int local_max = 0;
  for (int row = r0; row < r1; row++) {
    const uint4* g = reinterpret_cast<const uint4*>(src + (uint64_t)row * k);
    for (int q = tid; q < (k >> 4); q += kPrThreads) reinterpret_cast<uint4*>(row_s)[q] = __ldg(g + q);
    if (want_e && tid < r / 16)
      reinterpret_cast<uint4*>(es)[tid] = __ldg(reinterpret_cast<const uint4*>(E + (uint64_t)row * r) + tid);
    __syncthreads();
    if (dst) {
      // values stay in int8 without wrapping for |src| <= 64, |E| <= 32
      for (int q = tid; q < (k >> 4); q += kPrThreads) {
        const uint4 w = reinterpret_cast<const uint4*>(row_s)[q];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        uint32_t o[4];
#pragma unroll
        for (int v = 0; v < 4; v++) {
          uint32_t ov = 0;
#pragma unroll
          for (int b = 0; b < 4; b++) {
            const uint32_t pv = pn_s[16 * q + 4 * v + b];
            const int nv = (int)(int8_t)(ws[v] >> (8 * b)) + (int)es[(pv & 0xFFFFu) & (r - 1)] -
                           (int)es[(pv >> 16) & (r - 1)];
            ov |= (uint32_t)(uint8_t)(int8_t)nv << (8 * b);
          }
          o[v] = ov;
        }
        reinterpret_cast<uint4*>(dst + (uint64_t)row * k)[q] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (Pp) {
      int acc = 0;
      for (int i = pstart[j] + part; i < pstart[j + 1]; i += parts) acc += row_s[plist[i]];
      for (int i = mstart[j] + part; i < mstart[j + 1]; i += parts) acc -= row_s[mlist[i]];
      red[tid] = acc;
      __syncthreads();
      if (part == 0) {
        int v = 0;
        for (int qq = 0; qq < parts; qq++) v += red[qq * r + j];
        local_max = max(local_max, abs(v));
        if (corr && corr_off >= 0) {
          const uint64_t base = (uint64_t)row * 2 * r + corr_off + j;
          for (int li = 0; li < lmax; li++) {
            const int d = ((v + 64) & 127) - 64;
            corr[li * limb_stride + base] = (int8_t)d;
            v = (v - d) >> 7;
          }
        }
      }
    }
    if (want_e && corr && ecopy_off >= 0 && tid < r) {
      const int8_t e = es[tid];
      for (int li = 0; li < lmax; li++) corr[li * limb_stride + (uint64_t)row * 2 * r + ecopy_off + tid] = e;
    }
    __syncthreads();   // row_s, es and red are rewritten by the next row
  }
  if (Pp && maxabs) {
#pragma unroll
    for (int sft = 16; sft > 0; sft >>= 1) local_max = max(local_max, __shfl_xor_sync(0xffffffffu, local_max, sft));
    if ((tid & 31) == 0) atomicMax(maxabs, local_max);
  }
}

__global__ void __launch_bounds__(256) k_proj_matrix(const uint32_t* __restrict__ P, int k, int r,
                                                     int8_t* __restrict__ St) {
  const uint64_t total = (uint64_t)r * k;
  for (uint64_t i = (uint64_t)blockIdx.x * 256 + threadIdx.x; i < total; i += (uint64_t)gridDim.x * 256) {
    const uint32_t j = (uint32_t)(i / k), l = (uint32_t)(i - (uint64_t)j * k);
    const uint32_t p = P[l];
    St[i] = (int8_t)((int)((p & 0xFFFFu) == j) - (int)((p >> 16) == j));
  }
}

__global__ void __launch_bounds__(256) k_proj_corr(const int32_t* __restrict__ proj, int rows, int r,
                                                   int8_t* __restrict__ corr, int corr_off,
                                                   int32_t* __restrict__ maxabs, int lmax,
                                                   const int8_t* __restrict__ E, int ecopy_off) {
  const uint64_t limb_stride = (uint64_t)rows * 2 * r, total = (uint64_t)rows * r;
  int local_max = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * 256 + threadIdx.x; i < total; i += (uint64_t)gridDim.x * 256) {
    const uint64_t rr = i / r;
    const int j = (int)(i - rr * r);
    int v = proj[i];
    local_max = max(local_max, abs(v));
    if (corr) {
      for (int li = 0; li < lmax; li++) {
        const int d = ((v + 64) & 127) - 64;
        corr[li * limb_stride + rr * 2 * r + corr_off + j] = (int8_t)d;
        v = (v - d) >> 7;
      }
      if (E) {
        const int8_t e = E[i];
        for (int li = 0; li < lmax; li++) corr[li * limb_stride + rr * 2 * r + ecopy_off + j] = e;
      }
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) local_max = max(local_max, __shfl_xor_sync(0xffffffffu, local_max, s));
  if ((threadIdx.x & 31) == 0 && maxabs) atomicMax(maxabs, local_max);
}

// ------------------------------------------------------------------ C ABI
extern "C" {

uint64_t uwc_b3_scratch_words(uint64_t nbytes) {
  uint64_t nch = nbytes / 1024, words = 0;
  uint64_t cnt = (nch + kChunksPerCta - 1) / kChunksPerCta;
  words += 8 * cnt;
  while (cnt > (uint64_t)kReduceGroup) {
    cnt = (cnt + kReduceGroup - 1) / kReduceGroup;
    words += 8 * cnt;
  }
  return words < 8 ? 8 : words;
}

int uwc_b3_root_and_seed(const void* data, uint64_t nbytes, const uint32_t* key, const uint32_t* prefix,
                         const uint32_t* salt, uint32_t dim, uint32_t* root_out, uint32_t* seed_out,
                         uint32_t* scratch, uint64_t scratch_words, void* stream) {
  if (!data || !key || !scratch || (seed_out && (!prefix || !salt))) return UWC_ERR_ARG;
  if (nbytes == 0 || nbytes % 1024) return UWC_ERR_SHAPE;
  if (((uintptr_t)data) & 15) return UWC_ERR_ALIGN;
  if (scratch_words < uwc_b3_scratch_words(nbytes)) return UWC_ERR_SCRATCH;
  UWC_CHECK_DEVICE();
  cudaStream_t st = (cudaStream_t)stream;
  const uint64_t nch = nbytes / 1024;
  uint64_t cnt = (nch + kChunksPerCta - 1) / kChunksPerCta;
  k_b3_chunks<<<(unsigned)cnt, kChunksPerCta, 0, st>>>((const uint8_t*)data, nch, key, scratch, 1u);
  uwc_count_launch();
  uint32_t* cur = scratch;
  uint32_t* nxt = scratch + 8 * cnt;
  while (cnt > (uint64_t)kReduceGroup) {
    const uint64_t groups = (cnt + kReduceGroup - 1) / kReduceGroup;
    k_b3_reduce<<<(unsigned)groups, 512, 0, st>>>(cur, (uint32_t)cnt, key, nxt, 0, nullptr, nullptr, 0, nullptr,
                                                  nullptr, 1u);
    uwc_count_launch();
    cur = nxt;
    nxt += 8 * groups;
    cnt = groups;
  }
  k_b3_reduce<<<1, 512, 0, st>>>(cur, (uint32_t)cnt, key, nullptr, 1, prefix, salt, dim, root_out, seed_out, 1u);
  uwc_count_launch();
  return uwc_launch_status();
}

}  // extern "C"

int uwc_noise_uniform_zero2(int8_t* out, uint64_t nbytes, const uint32_t* label, const uint32_t* key,
                            int32_t* zero_me, int zero_n, int32_t* zero2, int zero2_n, void* stream) {
  if (!out || !label || !key || zero_n < 0 || (zero_n > 0 && !zero_me) || zero2_n < 0 || (zero2_n > 0 && !zero2))
    return UWC_ERR_ARG;
  if (nbytes % 32) return UWC_ERR_SHAPE;
  if (((uintptr_t)out) & 15) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  const uint64_t nblocks = nbytes / 32;
  if (nblocks > 0xFFFFFFFFull) return UWC_ERR_SHAPE;
  const uint64_t threads = std::max<uint64_t>(nblocks, (uint64_t)std::max(zero_n, zero2_n));
  if (threads == 0) return UWC_OK;
  k_noise_uniform<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(out, (uint32_t)nblocks, label,
                                                                                     key, zero_me, zero_n, zero2,
                                                                                     zero2_n);
  uwc_count_launch();
  return uwc_launch_status();
}

extern "C" {

int uwc_noise_uniform(int8_t* out, uint64_t nbytes, const uint32_t* label, const uint32_t* key, int32_t* zero_me,
                      int zero_n, void* stream) {
  return uwc_noise_uniform_zero2(out, nbytes, label, key, zero_me, zero_n, nullptr, 0, stream);
}

int uwc_noise_perm(uint32_t* out, uint32_t k, uint32_t r, const uint32_t* label, const uint32_t* key, void* stream) {
  if (!out || !label || !key) return UWC_ERR_ARG;
  if (r < 2 || (r & (r - 1)) || r > 65536) return UWC_ERR_SHAPE;
  UWC_CHECK_DEVICE();
  if (k == 0) return UWC_OK;
  const uint32_t nh = (k + 7) / 8;
  k_noise_perm<<<(nh + 127) / 128, 128, 0, (cudaStream_t)stream>>>(out, k, r, label, key);
  uwc_count_launch();
  return uwc_launch_status();
}

int uwc_noise_rows(const int8_t* src, int rows, int k, int r, const int8_t* E, const uint32_t* Pn, int8_t* dst,
                   const uint32_t* Pp, int8_t* corr, int corr_off, int ecopy_off, int32_t* maxabs, int lmax,
                   void* stream) {
  if (!src || (dst && (!E || !Pn)) || (ecopy_off >= 0 && corr && !E) || lmax < 0) return UWC_ERR_ARG;
  if (rows <= 0 || rows % kNrRows || k <= 0 || k % 16 || (r != 64 && r != 128 && r != 256)) return UWC_ERR_SHAPE;
  if (Pp && k > 65536) return UWC_ERR_SHAPE;   // the projection's index lists hold 16-bit columns
  if ((((uintptr_t)src) | ((uintptr_t)dst) | ((uintptr_t)Pn) | ((uintptr_t)Pp)) & 15) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  if (dst && !Pp) {
    const int grid = std::min(rows, uwc_num_sms() * kNaCtasPerSm);
    k_noise_add<<<grid, 256, 0, (cudaStream_t)stream>>>(src, rows, k, r, E, Pn, dst, corr, ecopy_off, lmax);
    uwc_count_launch();
    return uwc_launch_status();
  }
  // noising with a projection and / or an E copy: the fused gather kernel, one pass over the rows
  const int smem = k + (dst ? 4 * k : 0) + 4 * k + 4 * (4 * r + 2) + 256 + 4 * kPrThreads;
  if (smem > 227 * 1024) return UWC_ERR_SHAPE;
  static int smem_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && (dev < 0 || dev >= 64 || smem_set[dev] < smem)) {
    if (cudaFuncSetAttribute(k_noise_project, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
      cudaGetLastError();
      return UWC_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) smem_set[dev] = 227 * 1024;
  }
  const int per_sm = std::max(1, std::min(4, (200 * 1024) / std::max(smem, 1)));
  const int grid = std::min(rows, uwc_num_sms() * per_sm);
  k_noise_project<<<grid, kPrThreads, smem, (cudaStream_t)stream>>>(src, rows, k, r, E, Pn, dst, Pp, corr, corr_off,
                                                                    ecopy_off, maxabs, lmax);
  uwc_count_launch();
  return uwc_launch_status();
}

int uwc_proj_matrix(const uint32_t* P, int k, int r, int8_t* St, void* stream) {
  if (!P || !St) return UWC_ERR_ARG;
  if (k <= 0 || r <= 0) return UWC_ERR_SHAPE;
  UWC_CHECK_DEVICE();
  const uint64_t n = (uint64_t)r * k;
  const unsigned grid = (unsigned)std::min<uint64_t>(4096, (n + 255) / 256);
  k_proj_matrix<<<grid, 256, 0, (cudaStream_t)stream>>>(P, k, r, St);
  uwc_count_launch();
  return uwc_launch_status();
}

int uwc_proj_corr(const int32_t* proj, int rows, int r, int8_t* corr, int corr_off, int32_t* maxabs, int lmax,
                  void* stream) {
  return uwc_proj_corr_ecopy(proj, rows, r, corr, corr_off, maxabs, lmax, nullptr, -1, stream);
}

}  // extern "C"

int uwc_proj_corr_ecopy(const int32_t* proj, int rows, int r, int8_t* corr, int corr_off, int32_t* maxabs, int lmax,
                        const int8_t* E, int ecopy_off, void* stream) {
  if (!proj || lmax < 0 || (corr && corr_off < 0) || (E && (!corr || ecopy_off < 0))) return UWC_ERR_ARG;
  if (rows <= 0 || r <= 0) return UWC_ERR_SHAPE;
  UWC_CHECK_DEVICE();
  const uint64_t n = (uint64_t)rows * r;
  const unsigned grid = (unsigned)std::min<uint64_t>(4096, (n + 255) / 256);
  k_proj_corr<<<grid, 256, 0, (cudaStream_t)stream>>>(proj, rows, r, corr, corr_off, maxabs, lmax, E, ecopy_off);
  uwc_count_launch();
  return uwc_launch_status();
}

// ------------------------------------------------------------------ commitment without allocation
// Some callers cannot allocate device memory at the moment they commit to a matrix: code running
// while a CUDA graph is being captured (cudaMalloc is not a capturable operation), foreign-function
// callers (cgo, JNI, plain C) that own no device allocator and would otherwise have to manage a
// scratch buffer per device, and processes whose device memory is fully reserved up front by
// another framework's pool. uwc_b3_root_and_seed_noalloc serves them with a fixed scratch array
// in the library's own device memory instead of a caller buffer.
//
// Limit: the scratch holds the chaining values of up to kNoAllocMaxCtas chunk groups, i.e.
// inputs up to kNoAllocMaxBytes (128 MiB, one reduce level); larger inputs are rejected with
// UWC_ERR_SCRATCH. The array (32 KiB) lives on every GPU that loads the library until exit.
// All calls on a device share it and it keeps the last call's contents (every word the kernels
// read is written first in the same call, so nothing needs clearing); calls that overlap on the
// GPU (different streams, or concurrent host threads) race on it and must be serialized.
namespace {
constexpr uint64_t kNoAllocMaxCtas = kReduceGroup;                         // one final reduce level
constexpr uint64_t kNoAllocMaxBytes = kNoAllocMaxCtas * kChunksPerCta * 1024;  // 128 MiB
constexpr uint64_t kNoAllocWords = 8 * kNoAllocMaxCtas;

static __device__ __align__(256) uint32_t g_b3_noalloc_scratch[kNoAllocWords];

constexpr int kNoAllocDevices = 64;
std::atomic<uint32_t*> g_noalloc_ptr[kNoAllocDevices];
std::mutex g_noalloc_mu;

// Device address of the static scratch on the current device. The first call on a device looks
// it up with cudaGetSymbolAddress (with that device current) under a mutex, so host threads that
// make their first calls at the same time do not race; later calls read the cached address. In
// host code the array's name is only a stand-in and must never be passed to a kernel. The cache
// lives as long as the device's CUDA context: after cudaDeviceReset, uwc_b3_noalloc_forget()
// drops it so the next call looks the address up again.
int noalloc_scratch(uint32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  if (dev < 0 || dev >= kNoAllocDevices) return UWC_ERR_DEVICE;
  uint32_t* cached = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!cached) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    cached = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (!cached) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_b3_noalloc_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return UWC_ERR_CUDA;
      }
      cached = static_cast<uint32_t*>(p);
      g_noalloc_ptr[dev].store(cached, std::memory_order_release);
    }
  }
  *out = cached;
  return UWC_OK;
}
}  // namespace

extern "C" uint64_t uwc_b3_noalloc_max_bytes(void) { return kNoAllocMaxBytes; }

extern "C" void uwc_b3_noalloc_forget(void) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  for (int d = 0; d < kNoAllocDevices; d++) g_noalloc_ptr[d].store(nullptr, std::memory_order_release);
}

extern "C" int uwc_b3_root_and_seed_noalloc(const void* data, uint64_t nbytes, const uint32_t* key,
                                            const uint32_t* prefix, const uint32_t* salt, uint32_t dim,
                                            uint32_t* root_out, uint32_t* seed_out, void* stream) {
  if (!data || !key || (seed_out && (!prefix || !salt))) return UWC_ERR_ARG;
  if (nbytes == 0 || nbytes % 1024) return UWC_ERR_SHAPE;
  if (nbytes > kNoAllocMaxBytes) return UWC_ERR_SCRATCH;
  if (((uintptr_t)data) & 15) return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  uint32_t* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != UWC_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const uint64_t nch = nbytes / 1024;
  const uint64_t cnt = (nch + kChunksPerCta - 1) / kChunksPerCta;   // <= kNoAllocMaxCtas
  k_b3_chunks<<<(unsigned)cnt, kChunksPerCta, 0, st>>>((const uint8_t*)data, nch, key, scratch, 1u);
  uwc_count_launch();
  k_b3_reduce<<<1, 512, 0, st>>>(scratch, (uint32_t)cnt, key, nullptr, 1, prefix, salt, dim, root_out, seed_out, 1u);
  uwc_count_launch();
  return uwc_launch_status();
}
