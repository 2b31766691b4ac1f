// SHA-256 stage-output commitments on sm_100a (runtime/detgpu/sha.py): a stage's T output rows
// (float32) are committed as
//   row_root  = MerkleRoot(sha256(0x00 || block)) over the row's little-endian bytes in 1 KiB blocks
//   sout leaf = sha256(0x00 || "sout" || u32le t || row_root)
//   stage root = MerkleRoot(sout leaves)
// with RFC 6962 trees: node = sha256(0x01 || left || right), built bottom-up by pairing neighbours
// and promoting an odd last node, which is the same tree as RFC 6962's split at the largest power
// of two below n (runtime/detrt/stage.py:26-72, runtime/agent/proto.py:24-35). Only the roots (or
// 32 bytes per token) leave the GPU.
//
// SHA-256 is FIPS 180-4; the round constants and initial state below are its published values
// (the first 32 fraction bits of the cube / square roots of the first primes).
#include <algorithm>

#include "uwc_device.cuh"
#include "uwc_host.h"

namespace {

__constant__ const uint32_t kK[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
__constant__ const uint32_t kIV[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                      0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};

constexpr int kBlockWords = 256;   // 1 KiB row blocks (runtime/detrt/stage.py BLOCK)
constexpr int kMaxBlocks = 32;     // blocks per row held by one thread (rows up to 8192 floats)

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

// One SHA-256 compression of 16 big-endian message words into the state.
__device__ __forceinline__ void compress(uint32_t* st, const uint32_t* m) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; i++) w[i] = m[i];
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
  for (int i = 0; i < 64; i++) {
    if (i >= 16) {
      const uint32_t x = w[(i - 15) & 15], y = w[(i - 2) & 15];
      w[i & 15] += (rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3)) + w[(i - 7) & 15] + (rotr(y, 17) ^ rotr(y, 19) ^ (y >> 10));
    }
    const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + kK[i] + w[i & 15];
    const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d; st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

__device__ __forceinline__ void init(uint32_t* st) {
#pragma unroll
  for (int i = 0; i < 8; i++) st[i] = kIV[i];
}

// node = sha256(0x01 || l || r), digests as big-endian state words. The 65-byte message shifted
// by its one-byte prefix: word i = (S[i-1] << 24) | (S[i] >> 8) over S = l || r, S[-1] = 0x01.
__device__ void node(const uint32_t* l, const uint32_t* r, uint32_t* out) {
  uint32_t m[16], st[8];
  init(st);
  uint32_t prev = 0x01u;
#pragma unroll
  for (int i = 0; i < 16; i++) {
    const uint32_t s = i < 8 ? l[i] : r[i - 8];
    m[i] = (prev << 24) | (s >> 8);
    prev = s;
  }
  compress(st, m);
#pragma unroll
  for (int i = 0; i < 16; i++) m[i] = 0u;
  m[0] = (prev << 24) | (0x80u << 16);
  m[15] = 65u * 8u;
  compress(st, m);
#pragma unroll
  for (int i = 0; i < 8; i++) out[i] = st[i];
}

// sout leaf = sha256(0x00 || "sout" || u32le t || root): 41 bytes, one compression.
__device__ void sout_leaf(uint32_t t, const uint32_t* root, uint32_t* out) {
  uint32_t m[16], st[8];
  init(st);
  m[0] = 0x00736f75u;                                              // 0x00 's' 'o' 'u'
  m[1] = (0x74u << 24) | ((t & 0xffu) << 16) | (((t >> 8) & 0xffu) << 8) | ((t >> 16) & 0xffu);
  uint32_t prev = t >> 24;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    m[2 + i] = (prev << 24) | (root[i] >> 8);
    prev = root[i];
  }
  m[10] = (prev << 24) | (0x80u << 16);
#pragma unroll
  for (int i = 11; i < 15; i++) m[i] = 0u;
  m[15] = 41u * 8u;
  compress(st, m);
#pragma unroll
  for (int i = 0; i < 8; i++) out[i] = st[i];
}

// sha256(0x00 || block) of block bk of row r (one thread per block). The one-byte prefix shifts
// the little-endian data words: big-endian message word i is (d[i-1] byte 3, d[i] bytes 0..2).
__global__ void __launch_bounds__(128) k_block_leaves(const uint32_t* __restrict__ rows, int row_words, int nblk,
                                                      long long nrows, uint32_t* __restrict__ leaves) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nrows * nblk) return;
  const long long r = i / nblk;
  const int bk = (int)(i - r * nblk);
  const uint32_t* d = rows + r * row_words + (long long)bk * kBlockWords;
  const int nw = min(kBlockWords, row_words - bk * kBlockWords);   // data words of this block
  const uint32_t L = 1u + 4u * (uint32_t)nw;                       // message bytes
  const int nc = (int)((L + 8) / 64) + 1;                          // 64-byte chunks with padding
  uint32_t st[8];
  init(st);
  uint32_t prev = 0u;                                              // the 0x00 prefix as byte 3
  for (int c = 0; c < nc; c++) {
    uint32_t m[16];
#pragma unroll
    for (int w = 0; w < 16; w++) {
      const int j = 16 * c + w;
      const uint32_t cur = j < nw ? __ldg(d + j) : (j == nw ? 0x80u : 0u);   // 0x80 ends the message
      m[w] = __byte_perm(prev, cur, 0x3456);
      prev = cur;
    }
    if (c == nc - 1) {
      m[14] = 0u;
      m[15] = L * 8u;
    }
    compress(st, m);
  }
#pragma unroll
  for (int k = 0; k < 8; k++) leaves[i * 8 + k] = st[k];
}

// Per row: the Merkle root of its nblk block leaves (bottom-up, odd node promoted), then the sout
// leaf of token t = row % T.
__global__ void __launch_bounds__(64) k_sout_leaves(const uint32_t* __restrict__ leaves, int nblk, long long nrows,
                                                    int T, uint32_t* __restrict__ out) {
  const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= nrows) return;
  uint32_t lv[kMaxBlocks][8];
  for (int i = 0; i < nblk; i++)
#pragma unroll
    for (int k = 0; k < 8; k++) lv[i][k] = leaves[(r * nblk + i) * 8 + k];
  int n = nblk;
  while (n > 1) {
    int m = 0;
    for (int i = 0; i + 1 < n; i += 2, m++) node(lv[i], lv[i + 1], lv[m]);
    if (n & 1) {
#pragma unroll
      for (int k = 0; k < 8; k++) lv[m][k] = lv[n - 1][k];
      m++;
    }
    n = m;
  }
  sout_leaf((uint32_t)(r % T), lv[0], out + r * 8);
}

// One CTA per stage: the Merkle root of its T leaves, level by level, ping-ponging between the
// leaf buffer and a scratch buffer of the same size.
__global__ void __launch_bounds__(256) k_tree_roots(uint32_t* __restrict__ a, uint32_t* __restrict__ b, int n0,
                                                    uint32_t* __restrict__ roots) {
  uint32_t* src = a + (long long)blockIdx.x * n0 * 8;
  uint32_t* dst = b + (long long)blockIdx.x * n0 * 8;
  int n = n0;
  while (n > 1) {
    const int half = n >> 1;
    for (int i = threadIdx.x; i < half; i += blockDim.x) node(src + 16 * i, src + 16 * i + 8, dst + 8 * i);
    if ((n & 1) && threadIdx.x < 8) dst[8 * half + threadIdx.x] = src[8 * (n - 1) + threadIdx.x];
    __syncthreads();
    uint32_t* t = src;
    src = dst;
    dst = t;
    n = half + (n & 1);
  }
  if (threadIdx.x < 8) roots[blockIdx.x * 8 + threadIdx.x] = src[threadIdx.x];
}

int blocks_per_row(int D) { return std::max(1, (D + kBlockWords - 1) / kBlockWords); }

int launch_leaves(const float* rows, long long nrows, int D, int T, uint32_t* scratch, uint32_t* out,
                  cudaStream_t st) {
  const int nblk = blocks_per_row(D);
  const long long n = nrows * nblk;
  k_block_leaves<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(reinterpret_cast<const uint32_t*>(rows), D, nblk,
                                                               nrows, scratch);
  uwc_count_launch();
  k_sout_leaves<<<(unsigned)((nrows + 63) / 64), 64, 0, st>>>(scratch, nblk, nrows, T, out);
  uwc_count_launch();
  return uwc_launch_status();
}

}  // namespace

extern "C" uint64_t uwc_stage_scratch_words(long long nrows, int D) {
  if (nrows <= 0 || D < 0) return 0;
  return (uint64_t)nrows * blocks_per_row(D) * 8 + (uint64_t)nrows * 16;
}

extern "C" int uwc_stage_out_leaves(const float* rows, long long nrows, int D, int T, uint32_t* scratch,
                                    uint64_t scratch_words, uint32_t* leaves, void* stream) {
  if (!rows || !scratch || !leaves || nrows < 0 || D < 0 || T <= 0) return UWC_ERR_ARG;
  if (blocks_per_row(D) > kMaxBlocks || nrows % T) return UWC_ERR_SHAPE;
  if (scratch_words < uwc_stage_scratch_words(nrows, D)) return UWC_ERR_SCRATCH;
  UWC_CHECK_DEVICE();
  if (nrows == 0) return UWC_OK;
  return launch_leaves(rows, nrows, D, T, scratch, leaves, (cudaStream_t)stream);
}

extern "C" int uwc_stage_roots(const float* rows, int B, int T, int D, uint32_t* scratch, uint64_t scratch_words,
                               uint32_t* roots, void* stream) {
  if (!rows || !scratch || !roots || B < 0 || T <= 0 || D < 0) return UWC_ERR_ARG;
  if (blocks_per_row(D) > kMaxBlocks) return UWC_ERR_SHAPE;
  const long long nrows = (long long)B * T;
  if (scratch_words < uwc_stage_scratch_words(nrows, D)) return UWC_ERR_SCRATCH;
  UWC_CHECK_DEVICE();
  if (B == 0) return UWC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  uint32_t* blk = scratch;                                          // nrows * nblk * 8
  uint32_t* lv = scratch + (uint64_t)nrows * blocks_per_row(D) * 8; // nrows * 8 (sout leaves)
  uint32_t* pp = lv + (uint64_t)nrows * 8;                           // nrows * 8 (tree ping-pong)
  int rc = launch_leaves(rows, nrows, D, T, blk, lv, st);
  if (rc != UWC_OK) return rc;
  k_tree_roots<<<B, 256, 0, st>>>(lv, pp, T, roots);
  uwc_count_launch();
  return uwc_launch_status();
}
