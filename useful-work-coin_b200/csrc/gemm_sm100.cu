// The NoisyGEMM on Blackwell tensor cores (sm_100a): C = A B^T, int8 x int8 -> int32 with
// tcgen05.mma kind::i8, TMEM accumulators and TMA-fed 128-byte-swizzled shared-memory stages.
//
// Reference semantics: noisy_gemm (miner/ampere/uwc_ampere/kernels.cu:482-715), launched by
// ops.gemm (ops.py:185-198). Five schedules share one persistent, warp-specialized kernel,
// specialized at compile time on the schedule and on the hash chunk width r:
//
//   MODE_MINE      FLAG_HASH without an output (MinedWeight.noise_mine, ops.py:349-364). A work
//                  unit is a 256 x 256 output block held as two 128 x 256 TMEM accumulators X (rows
//                  0-127) and Y (rows 128-255) sharing the B tile. Per r-column chunk of k the MMA
//                  warp issues X then Y, so each accumulator's running sum is read by the epilogue
//                  while the tensor core works on the other.
//   MODE_MINE_FWD  FLAG_HASH with an output (MinedWeight.forward, ops.py:316-347): the mining
//                  schedule, and in the same kernel the output. At the last snapshot, already in
//                  registers for the hash, each thread stores its raw int32 row (into its own output
//                  row, or a per-CTA staging block for bf16). With FLAG_DENOISE the freed accumulator
//                  then receives the correction R = sum_li 128^li corrA[li] corrB[li]^T by Horner
//                  steps (the epilogue shifts R by 7 bits in TMEM between limbs) and the thread
//                  writes out = raw - R, scaled; without it, the scaled raw row. The raw row is
//                  reread by the thread that wrote it microseconds earlier (from L2), never as an
//                  m x n matrix pass over HBM.
//   MODE_FWD       FLAG_DENOISE without FLAG_HASH (MinedWeight.forward with hash_tiles=False).
//                  A unit is a 128 x 256 block held as two 128 x 128 accumulators (column halves)
//                  plus a 128 x 256 correction accumulator R built before the main loop (Horner).
//                  The output is acc - R, exact in int32.
//   MODE_CORR      the scaling pass of a split-K plain GEMM with an fp32 / bf16 output: out =
//                  scale(acc) with acc read back from the summed int32 partials.
//   MODE_PLAIN     no flags: a 128 x 256 block per unit, two accumulators used alternately across
//                  units so the store of one unit overlaps the main loop of the next.
//
// The MMA issue loop is fully unrolled per 128-byte k-block stage: the tensor core only runs at
// its rate when tcgen05.mma instructions are issued back to back.
//
// Hash tiles (pearl_glue.py:14-15): rows g + 8i (i < 8), cols 2t + {0,1} + 8j (j < 8) of a
// 64 x 64 block. An epilogue warp reads its TMEM quadrant (32 rows) x 64 columns with
// tcgen05.ld.32x32b (thread = row, registers = consecutive columns), XORs each row's values
// into four partials by t = (col / 2) % 4, then a 3-shuffle reduce-scatter over the lanes of
// rows g, g+8, g+16, g+24 leaves lane (g + 8t) with tile (g, t)'s XOR over the quadrant.
// Rows 32-63 of a 64-row block live in the next quadrant (the next warp). XOR and rotl are linear
// over GF(2): the reference's msg[c % 16] = rotl(msg[c % 16], 13) ^ x_c equals the XOR over the
// chunks of slot s of rotl(x_c, 13 * (updates of slot s after c)). So every epilogue thread
// pre-rotates its chunk contribution and XOR-reduces it into the unit's message buffer in shared
// memory (red.shared.xor; 512 tiles x 16 words = 32 KiB): no message state in registers, no
// traffic to L2 (reductions into global memory cost a third of the kernel's time at r = 64,
// measured), and the two quadrant halves of a tile combine in the same word. Two CTA-wide
// hand-offs per unit order the reductions before the tile hashes and the hashes (which clear the
// words) before the next unit's reductions.
//
// Warp roles (576 threads, one CTA per SM, all 512 TMEM columns):
//   0..15   epilogue: warp w reads TMEM lanes 32*(w%4).. and the 64-column block w/4; at the end
//           of a hashed unit each of the 512 threads hashes one tile (keyed BLAKE3 of its message,
//           target compare, win record), so the hash work is spread over all four SM sub-partitions
//   16      TMA producer (one elected lane issues)
//   17      MMA issuer (one lane issues); allocates and frees TMEM
#include <algorithm>
#include <atomic>

#include "det_math.cuh"
#include "uwc_device.cuh"
#include "uwc_host.h"

namespace {

enum Mode { MODE_PLAIN = 0, MODE_MINE = 1, MODE_FWD = 2, MODE_CORR = 3, MODE_MINE_FWD = 4 };

constexpr int kEpiWarps = 16;
constexpr int kProducerWarp = kEpiWarps;               // 16
constexpr int kMmaWarp = kProducerWarp + 1;             // 17
constexpr int kThreads = (kMmaWarp + 1) * 32;           // 576
constexpr int kKB = 128;                                // K bytes per stage (one 128-byte swizzle row)
constexpr int kUN = 256;                                // output columns per unit
constexpr int kMaxTiles = 512;                          // hash tiles per unit (MINE)
constexpr int kMsgWords = kMaxTiles * 16;               // one unit's tile messages (32 KiB, shared memory)
constexpr int kStageWords = 2 * kEpiWarps * 32 * 64;   // a unit's raw products: 2 accumulators x 512 threads x 64
constexpr int kBarBytes = 256;

// The epilogue's tensor-memory hand-offs (accumulator free, R shifted, R consumed) order only TMEM
// accesses, so they arrive relaxed: a releasing arrive would first wait for the thread's earlier
// output stores and message reductions, holding the tensor core back (measured at r = 64).
#define ACC_ARRIVE mbar_arrive_relaxed

struct Params {
  int m, n, k, r;
  int hash;         // FLAG_HASH
  int denoise;      // FLAG_DENOISE
  int lmax;
  int out_mode;
  int max_wins;
  int nm, nn, nunits;
  int nsplit, kps;         // PLAIN split-K: k-block ranges per unit (nsplit 1 = whole k)
  const int32_t* maxabs;
  const uint32_t* key;
  const uint32_t* target;
  uint32_t* wins;
  int32_t* stage;          // MODE_MINE_FWD: per CTA kStageWords int32 (the unit's raw products, thread-interleaved)
  const int32_t* acc_in;   // MODE_CORR: the summed int32 split-K product, m x n
  const float* a_scale;
  const float* b_scale;
  void* out;
  uint32_t* status;
  uint32_t one;      // 1, opaque to the compiler (multiply-add additions in the tile hash)
  uint64_t wait_ns;  // bound of every wait (1 s; shortened by the test hook)
  int withhold;      // test hook: the producer issues no copies, so the first wait runs out
  // Batched PLAIN launches (nbatch > 1 or causal): batch bt reads A rows bt * a_brows + [0, m) and
  // B rows (bt / b_bdiv) * b_brows + [0, n), and writes its m x n int32 block at out + bt * m * n.
  // causal 1 (Q K^T): block (m0, n0) runs only if some row t in [m0, m0 + 128) sees a column of it
  // (column j visible to row t when j <= cshift + t). causal 2 (P V, A = [P_hi; P_lo] rows of qrows
  // each): the k range stops after the last key row (m0 % qrows) + 127 sees.
  int nbatch, b_bdiv, causal, cshift, qrows, units_per_batch;
  long long a_brows, b_brows;
  // PLAIN fused output steps (uwc_gemm_epi): F32 out + resid (m x n fp32) when resid is set; with
  // swiglu, B is [gate; up] (2n rows), a unit's 256 B rows are 128 gate rows over the matching up
  // rows, and out (m x n fp32) = det_silu(deq(gate)) * deq(up) (b_scale in B's row order)
  const float* resid;
  int swiglu;
};

// R: hash chunk width in k (64, 128, 256), or 0 for no hashing.
template <int MODE, int R>
struct Cfg {
  static constexpr bool HASH = R != 0;
  static constexpr bool MINE = MODE == MODE_MINE || MODE == MODE_MINE_FWD;   // the mining schedule
  static constexpr int UM = MINE ? 256 : 128;                    // output rows per unit
  static constexpr int NACC = MODE == MODE_PLAIN ? 1 : 2;
  static constexpr int ACC_N = MODE == MODE_FWD ? 128 : 256;    // MMA N per accumulator
  static constexpr bool CORR = MODE == MODE_FWD || MODE == MODE_CORR;  // R built before the main loop
  static constexpr int A_BYTES = UM * kKB;
  static constexpr int STAGE = A_BYTES + kUN * kKB;              // 64 KiB (MINE) / 48 KiB
  static constexpr int NST = MINE || MODE == MODE_PLAIN ? 3 : (MODE == MODE_CORR ? 2 : 4);
  // Per epilogue warp a padded 32 x 33-word shared-memory tile that turns thread-per-row data into
  // row-contiguous global accesses (MODE_CORR's read-back and stores, MODE_PLAIN's stores).
  static constexpr int TILE_WORDS = 32 * 33;
  static constexpr int TILE_BYTES = MODE == MODE_CORR || MODE == MODE_PLAIN ? kEpiWarps * TILE_WORDS * 4 : 0;
  static constexpr int MSG_BYTES = HASH ? kMsgWords * 4 : 0;     // the unit's tile messages
  static constexpr int SMEM = NST * STAGE + TILE_BYTES + MSG_BYTES + kBarBytes + 1024;  // +1024: alignment
  static constexpr int PARTS = R == 64 ? 2 : 1;                  // chunks per stage
  static constexpr int SPAN = R == 256 ? 2 : 1;                  // stages per chunk
  static constexpr int ACC_WARPS = MODE == MODE_FWD ? kEpiWarps / 2 : kEpiWarps;  // readers per acc
};

struct Bars;
struct Bars {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t acc_full[4];
  uint64_t acc_empty[4];
  uint64_t r_full, r_scaled, r_empty;
  uint64_t c_ready[2];      // MODE_MINE_FWD, per accumulator: a Horner step of R has landed in TMEM
  uint64_t c_shifted[2];    // MODE_MINE_FWD, per accumulator: the epilogue shifted R by 7 bits
  uint64_t hash_ready;      // every epilogue thread's XOR reductions of the unit landed
  uint64_t hash_done;       // every tile of the unit hashed and its message words cleared
  uint64_t tiles_done;      // MINE_FWD: the output pass's transpose tiles (in the message buffer) re-zeroed
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int L;
};
static_assert(sizeof(Bars) <= kBarBytes, "barrier block");

__device__ __forceinline__ void unit_coords(const Params& p, int u, int UM, int& m0, int& n0) {
  constexpr int G = 16;  // group of row blocks that sweep the columns together (L2 reuse of B)
  const int grp = G * p.nn, gid = u / grp, first = gid * G;
  const int gsz = min(p.nm - first, G), in = u - gid * grp;
  m0 = (first + in % gsz) * UM;
  n0 = (in / gsz) * kUN;
}

// Causal Q K^T: the column blocks row block mb needs (the first n0 past cshift + mb*128 + 127 is out).
__device__ __forceinline__ int causal_nblocks(const Params& p, int mb) {
  return min(p.nn, (p.cshift + mb * 128 + 128 + kUN - 1) / kUN);
}

// Unit u of a split-K PLAIN launch: output block (unit_coords of u % (nm * nn)) and the k-block
// range [kb0, kb0 + nkb) of split u / (nm * nn). Without splitting, the whole k. Batched
// launches: batch bt = u / units_per_batch, then the block within the batch (causal: row blocks
// in order, each with its visible column blocks).
__device__ __forceinline__ void unit_span(const Params& p, int u, int UM, int kblocks, int& m0, int& n0, int& kb0,
                                          int& nkb, int& bt) {
  bt = 0;
  if (p.units_per_batch > 0) {
    bt = u / p.units_per_batch;
    int r = u - bt * p.units_per_batch;
    kb0 = 0;
    nkb = kblocks;
    if (p.causal == 1) {
      int mb = 0;
      for (; mb + 1 < p.nm; mb++) {
        const int c = causal_nblocks(p, mb);
        if (r < c) break;
        r -= c;
      }
      m0 = mb * 128;
      n0 = r * kUN;
      return;
    }
    m0 = (r % p.nm) * 128;
    n0 = (r / p.nm) * kUN;
    if (p.causal == 2) nkb = min(kblocks, (p.cshift + m0 % p.qrows + 128 + kKB - 1) / kKB);
    return;
  }
  if (p.nsplit > 1) {
    const int nmn = p.nm * p.nn, ks = u / nmn;
    unit_coords(p, u - ks * nmn, UM, m0, n0);
    kb0 = ks * p.kps;
    nkb = min(kblocks - kb0, p.kps);
  } else {
    unit_coords(p, u, UM, m0, n0);
    kb0 = 0;
    nkb = kblocks;
  }
}

// Limb count from the projections' max |value| (kernels.cu:602-607 thresholds), capped at lmax.
__device__ __forceinline__ int limbs_from_maxabs(const Params& p) {
  if (!p.denoise) return 0;
  const int mx = max(p.maxabs[0], p.maxabs[1]);
  int L = 1;
  if (mx > 63) L = 2;
  if (mx > 8127) L = 3;
  if (mx > 1040319) L = 4;
  return min(L, p.lmax);
}

// ------------------------------------------------------------------ output stores
__device__ __forceinline__ uint32_t bf16_rne(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

// Store 32 consecutive int32 accumulators of one row (columns c0..c0+31) in the chosen format.
__device__ __forceinline__ void store_row32(const Params& p, int row, int c0, const int32_t* v) {
  if (p.out_mode == UWC_OUT_NONE || row >= p.m || c0 >= p.n) return;
  const bool full = c0 + 32 <= p.n;
  if (p.out_mode == UWC_OUT_I32 || p.out_mode == UWC_OUT_F32) {
    uint32_t w[32];
    if (p.out_mode == UWC_OUT_I32) {
#pragma unroll
      for (int i = 0; i < 32; i++) w[i] = (uint32_t)v[i];
    } else {
      const float sx = p.a_scale[row];
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const float sw = (c0 + i < p.n) ? __ldg(p.b_scale + c0 + i) : 0.f;
        w[i] = __float_as_uint(__fmul_rn(__fmul_rn(__int2float_rn(v[i]), sx), sw));
      }
    }
    uint32_t* o = reinterpret_cast<uint32_t*>(p.out) + (uint64_t)row * p.n + c0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 8; i++)
        reinterpret_cast<uint4*>(o)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; i++)
        if (c0 + i < p.n) o[i] = w[i];
    }
  } else {  // UWC_OUT_BF16: RNE((float(acc) * a_scale) * b_scale)
    const float sx = p.a_scale[row];
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float s0 = (c0 + 2 * i < p.n) ? __ldg(p.b_scale + c0 + 2 * i) : 0.f;
      const float s1 = (c0 + 2 * i + 1 < p.n) ? __ldg(p.b_scale + c0 + 2 * i + 1) : 0.f;
      const float f0 = __fmul_rn(__fmul_rn(__int2float_rn(v[2 * i]), sx), s0);
      const float f1 = __fmul_rn(__fmul_rn(__int2float_rn(v[2 * i + 1]), sx), s1);
      w[i] = bf16_rne(f0) | (bf16_rne(f1) << 16);
    }
    uint16_t* o = reinterpret_cast<uint16_t*>(p.out) + (uint64_t)row * p.n + c0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 4; i++)
        reinterpret_cast<uint4*>(o)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; i++)
        if (c0 + i < p.n) o[i] = (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
    }
  }
}

// Four consecutive outputs of one row (c % 4 == 0, n % 4 == 0) in the chosen format.
__device__ __forceinline__ void store4(const Params& p, int row, int c, int32_t v0, int32_t v1, int32_t v2, int32_t v3) {
  if (p.out_mode == UWC_OUT_I32) {
    *reinterpret_cast<int4*>(static_cast<int32_t*>(p.out) + (uint64_t)row * p.n + c) = make_int4(v0, v1, v2, v3);
    return;
  }
  const float sx = p.a_scale[row];
  const float f0 = __fmul_rn(__fmul_rn(__int2float_rn(v0), sx), __ldg(p.b_scale + c));
  const float f1 = __fmul_rn(__fmul_rn(__int2float_rn(v1), sx), __ldg(p.b_scale + c + 1));
  const float f2 = __fmul_rn(__fmul_rn(__int2float_rn(v2), sx), __ldg(p.b_scale + c + 2));
  const float f3 = __fmul_rn(__fmul_rn(__int2float_rn(v3), sx), __ldg(p.b_scale + c + 3));
  if (p.out_mode == UWC_OUT_F32) {
    float4 o = make_float4(f0, f1, f2, f3);
    if (p.resid) {
      const float4 x = *reinterpret_cast<const float4*>(p.resid + (uint64_t)row * p.n + c);
      o = make_float4(__fadd_rn(x.x, f0), __fadd_rn(x.y, f1), __fadd_rn(x.z, f2), __fadd_rn(x.w, f3));
    }
    *reinterpret_cast<float4*>(static_cast<float*>(p.out) + (uint64_t)row * p.n + c) = o;
  } else {
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + (uint64_t)row * p.n + c) =
        make_uint2(bf16_rne(f0) | (bf16_rne(f1) << 16), bf16_rne(f2) | (bf16_rne(f3) << 16));
  }
}

// ------------------------------------------------------------------ hash-tile fold
// XOR the 32 values of one row (consecutive columns) into four partials by t = (col / 2) % 4.
__device__ __forceinline__ void fold_row32(const uint32_t* v, uint32_t* pt) {
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const int b = 2 * t;
    pt[t] ^= (v[b] ^ v[b + 1] ^ v[b + 8]) ^ (v[b + 9] ^ v[b + 16] ^ v[b + 17]) ^ (v[b + 24] ^ v[b + 25]);
  }
}

// f ? if1 : if0 for f in {0, 1}, as two multiply-adds: the selects of the reduce-scatter run on
// the FMA pipe, next to the XOR fold that saturates the integer ALU pipe.
__device__ __forceinline__ uint32_t imad_sel(uint32_t if1, uint32_t if0, uint32_t f) {
  uint32_t d, r;
  asm("mad.lo.u32 %0, %1, 0xFFFFFFFF, %2;" : "=r"(d) : "r"(if0), "r"(if1));
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(d), "r"(f), "r"(if0));
  return r;
}

// Reduce-scatter over the lanes of rows g, g+8, g+16, g+24 (lane bits 3 and 4): lane (g + 8t)
// ends with the XOR of partial t over those four rows. Each step sends the half the partner keeps
// and recovers its own half as (both halves) ^ (sent half).
__device__ __forceinline__ uint32_t reduce_scatter4(const uint32_t* pt, int lane) {
  const uint32_t f4 = (lane >> 4) & 1, f3 = (lane >> 3) & 1;
  const uint32_t send_a = imad_sel(pt[0], pt[2], f4), send_b = imad_sel(pt[1], pt[3], f4);
  const uint32_t k0 = pt[0] ^ pt[2] ^ send_a ^ __shfl_xor_sync(0xffffffffu, send_a, 16);
  const uint32_t k1 = pt[1] ^ pt[3] ^ send_b ^ __shfl_xor_sync(0xffffffffu, send_b, 16);
  const uint32_t send = imad_sel(k0, k1, f3);
  return k0 ^ k1 ^ send ^ __shfl_xor_sync(0xffffffffu, send, 8);
}

// XOR into a shared-memory word (the tile messages of the unit being mined).
__device__ __forceinline__ void red_xor_shared(uint32_t* addr, uint32_t v) {
  asm volatile("red.shared.xor.b32 [%0], %1;" ::"r"(smem_u32(addr)), "r"(v) : "memory");
}

// Keyed BLAKE3 of hash tile `slot` of a finished unit's message buffer (shared memory), target
// compare and win record (kernels.cu:574-596). Slot bits: lane-in-group (5), 64-column block (2),
// 64-row half (1), 128-row accumulator (1); the message words of a slot are kMaxTiles apart.
// Clears the words for the next unit.
__device__ __forceinline__ void hash_tile(const Params& p, uint32_t* msg, int m0, int n0, int slot) {
  const int ln = slot & 31, cbk = (slot >> 5) & 3, rb = (slot >> 7) & 1, a = slot >> 8;
  uint32_t w[16], hv[8], key[8];
#pragma unroll
  for (int i = 0; i < 16; i++) {
    w[i] = msg[i * kMaxTiles + slot];
    msg[i * kMaxTiles + slot] = 0u;
  }
  if (m0 + a * 128 + rb * 64 >= p.m || n0 + cbk * 64 >= p.n) return;
#pragma unroll
  for (int i = 0; i < 8; i++) key[i] = __ldg(p.key + i);
  b3::hash64<true>(key, w, hv, p.one);
  bool le = true, decided = false;
#pragma unroll
  for (int i = 7; i >= 0; i--) {
    const uint32_t t = __ldg(p.target + i);
    if (!decided && hv[i] != t) {
      le = hv[i] < t;
      decided = true;
    }
  }
  if (le) {
    const uint32_t ws = atomicAdd(p.wins, 1u);
    if (ws < (uint32_t)p.max_wins) {
      uint32_t* rec = p.wins + 1 + (uint64_t)ws * UWC_WIN_WORDS;
      rec[0] = (uint32_t)(m0 + a * 128 + rb * 64 + (ln >> 2));
      rec[1] = (uint32_t)(n0 + cbk * 64 + 2 * (ln & 3));
#pragma unroll
      for (int i = 0; i < 8; i++) rec[2 + i] = hv[i];
    }
  }
}

// A thread's 64 raw values (both halves of its last snapshot) into the CTA's staging block,
// thread-interleaved: quad i of thread T at uint4 index i * 512 + T, so every store instruction of a
// warp writes 512 contiguous bytes (a row-major store would touch 32 lines per instruction).
__device__ __forceinline__ void store_raw64(uint4* stage, int tid, const uint32_t* v, const uint32_t* v2) {
#pragma unroll
  for (int i = 0; i < 8; i++) stage[i * 512 + tid] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
#pragma unroll
  for (int i = 0; i < 8; i++)
    stage[(8 + i) * 512 + tid] = make_uint4(v2[4 * i], v2[4 * i + 1], v2[4 * i + 2], v2[4 * i + 3]);
}

// 16 int32 of one row (columns c0..c0+15) converted in place to the output words: I32 as is, F32
// the detrt dequant, BF16 packed pairs in w[0..7]. Returns the number of 16-byte quads (4 or 2).
__device__ __forceinline__ int convert16(const Params& p, int row, int c0, uint32_t* w) {
  if (p.out_mode == UWC_OUT_I32) return 4;
  const float sx = row < p.m ? p.a_scale[row] : 0.f;
  if (p.out_mode == UWC_OUT_F32) {
#pragma unroll
    for (int i = 0; i < 16; i++)
      w[i] = __float_as_uint(__fmul_rn(__fmul_rn(__int2float_rn((int32_t)w[i]), sx), __ldg(p.b_scale + c0 + i)));
    return 4;
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float f0 = __fmul_rn(__fmul_rn(__int2float_rn((int32_t)w[2 * i]), sx), __ldg(p.b_scale + c0 + 2 * i));
    const float f1 = __fmul_rn(__fmul_rn(__int2float_rn((int32_t)w[2 * i + 1]), sx), __ldg(p.b_scale + c0 + 2 * i + 1));
    w[i] = bf16_rne(f0) | (bf16_rne(f1) << 16);
  }
  return 2;
}

// Warp-wide bounded wait: every lane polls the barrier (measured faster to wake than one polling
// lane plus a warp sync) and the warp agrees on the verdict.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint32_t* status,
                                          uint64_t wait_ns) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, status, wait_ns));
}

template <int MODE, int R>
__global__ void __launch_bounds__(kThreads, 1)
    k_noisy_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmCA, const __grid_constant__ CUtensorMap tmCB, const Params p) {
  using C = Cfg<MODE, R>;
  constexpr bool FWDH = MODE == MODE_MINE_FWD;   // the hashed forward: output (and correction) in the same pass
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* const tiles = reinterpret_cast<uint32_t*>(smem + C::NST * C::STAGE);
  uint32_t* const msg = reinterpret_cast<uint32_t*>(smem + C::NST * C::STAGE + C::TILE_BYTES);
  Bars* bars = reinterpret_cast<Bars*>(smem + C::NST * C::STAGE + C::TILE_BYTES + C::MSG_BYTES);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NST; s++) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], C::ACC_WARPS);
      mbar_init(&bars->c_ready[a], 1);
      mbar_init(&bars->c_shifted[a], kEpiWarps);
    }
    // message hand-offs are signalled by every epilogue thread (arrival counts in threads)
    mbar_init(&bars->hash_ready, kEpiWarps * 32);
    mbar_init(&bars->hash_done, kEpiWarps * 32);
    mbar_init(&bars->tiles_done, kEpiWarps * 32);
    mbar_init(&bars->r_full, 1);
    mbar_init(&bars->r_scaled, kEpiWarps);
    mbar_init(&bars->r_empty, kEpiWarps);
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    bars->L = C::CORR || FWDH ? limbs_from_maxabs(p) : 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  if (C::HASH && warp < kEpiWarps) {
    uint4* z = reinterpret_cast<uint4*>(msg);
    for (int i = threadIdx.x; i < kMsgWords / 4; i += kEpiWarps * 32) z[i] = make_uint4(0, 0, 0, 0);
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if ((C::CORR || FWDH) && p.denoise) {
      tma_prefetch_desc(&tmCA);
      tma_prefetch_desc(&tmCB);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const int L = bars->L;
  const int k = p.k;
  const int kblocks = MODE == MODE_CORR ? 0 : (k + kKB - 1) / kKB;
  const int nch = C::HASH ? k / R : 1;                         // snapshots per accumulator per unit
  const int cblocks = C::CORR || FWDH ? (2 * p.r) / kKB : 1;  // k-blocks per correction limb

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp runs the schedule (loop state stays warp-uniform, off the vector ALU that
    // the epilogue saturates); one elected lane issues the copies.
    {
      const bool leader = elect_one();
      uint32_t gk = 0;
      // (test hook: with `withhold` no copy is issued and the MMA warp's first wait runs out)
      for (int u = blockIdx.x; u < p.nunits && !p.withhold && !__any_sync(0xffffffffu, *abort_flag); u += gridDim.x) {
        int m0, n0, kb0, nkb, bt;
        unit_span(p, u, C::UM, kblocks, m0, n0, kb0, nkb, bt);
        // correction blocks: before the main loop (FWD, CORR) or after it (MINE_FWD)
        const int ncorr = C::CORR ? L * cblocks : 0;
        const int npost = FWDH ? L * cblocks : 0;
        const int nblk = ncorr + nkb + npost;
        for (int b = 0; b < nblk; b++, gk++) {
          const int s = gk % C::NST;
          const uint32_t ph = (gk / C::NST) & 1;
          if (!warp_wait(&bars->empty[s], ph ^ 1, abort_flag, p.status, p.wait_ns)) break;
          uint8_t* sA = smem + s * C::STAGE;
          uint8_t* sB = sA + C::A_BYTES;
          if (!leader) continue;
          mbar_expect_tx(&bars->full[s], C::STAGE);
          if (b < ncorr || b >= ncorr + nkb) {
            const int bb = b < ncorr ? b : b - ncorr - nkb;
            const int li = L - 1 - bb / cblocks, kb = bb % cblocks;
            tma_load_2d(sA, &tmCA, &bars->full[s], kb * kKB, li * p.m + m0);
            tma_load_2d(sB, &tmCB, &bars->full[s], kb * kKB, li * p.n + n0);
          } else {
            const int kb = kb0 + b - ncorr;
            tma_load_2d(sA, &tmA, &bars->full[s], kb * kKB, (int)(bt * p.a_brows) + m0);
            if (p.swiglu) {
              // 128 gate rows, then their 128 up rows (tmCB: B with 128-row boxes)
              tma_load_2d(sB, &tmCB, &bars->full[s], kb * kKB, n0 / 2);
              tma_load_2d(sB + 128 * kKB, &tmCB, &bars->full[s], kb * kKB, p.n + n0 / 2);
            } else {
              tma_load_2d(sB, &tmB, &bars->full[s], kb * kKB, (int)((bt / p.b_bdiv) * p.b_brows) + n0);
            }
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // As for the producer: the whole warp waits and keeps the schedule, one elected lane issues
    // the MMAs and commits.
    {
      const bool leader = elect_one();
      uint32_t gk = 0;                      // k-blocks consumed (ring position)
      uint32_t snaps[2] = {0, 0};           // snapshots produced per accumulator
      uint32_t writes[2] = {0, 0};          // MINE: waits for a free accumulator (snapshots + corrections)
      uint32_t shifted[2] = {0, 0};         // MINE_FWD: waits for the epilogue's Horner shifts
      uint32_t r_scaled_waits = 0;
      int local = 0;
      bool ok = true;
      const uint32_t smem_base = smem_u32(smem);
      constexpr uint32_t id_acc = idesc_i8(128, C::ACC_N);
      for (int u = blockIdx.x; u < p.nunits && ok; u += gridDim.x, local++) {
        int m0, n0, kb0, nkb, bt;
        unit_span(p, u, C::UM, kblocks, m0, n0, kb0, nkb, bt);
        // ---- correction accumulator R (FWD): Horner over limbs, highest limb first
        if (C::CORR && L > 0) {
          // MODE_CORR with up to two limbs keeps each limb's product in its own 256 columns (the
          // epilogue adds them as P0 + (P1 << 7)); otherwise Horner steps in columns 256..511
          const bool direct = MODE == MODE_CORR && L <= 2;
          for (int li = L - 1; li >= 0 && ok; li--) {
            const uint32_t tR = tmem + (direct ? 256 * li : 256);
            if (li == L - 1)
              ok = warp_wait(&bars->r_empty, (local & 1) ^ 1, abort_flag, p.status, p.wait_ns);
            else if (!direct)
              ok = warp_wait(&bars->r_scaled, r_scaled_waits++ & 1, abort_flag, p.status, p.wait_ns);
            if (!ok) break;
            tc_fence_after();
            for (int kb = 0; kb < cblocks && ok; kb++, gk++) {
              const int s = gk % C::NST;
              ok = warp_wait(&bars->full[s], (gk / C::NST) & 1, abort_flag, p.status, p.wait_ns);
              if (!ok) break;
              tc_fence_after();
              const uint32_t aA = smem_base + s * C::STAGE, aB = aA + C::A_BYTES;
              const uint64_t ad = sdesc_sw128(aA), bd = sdesc_sw128(aB);
              if (leader) {
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
                  mma_i8(tR, ad + 2 * ks, bd + 2 * ks, idesc_i8(128, 256),
                         ((direct || li == L - 1) && kb == 0 && ks == 0) ? 0u : 1u);
              }
              if (leader) mma_commit(&bars->empty[s]);
            }
            if (leader && (!direct || li == 0)) mma_commit(&bars->r_full);
          }
        }
        // ---- main loop, one 128-column k-block stage at a time, MMAs issued back to back
        const int nacc = (C::MINE && m0 + 128 >= p.m) ? 1 : C::NACC;
        const int pbuf = local & 1;   // PLAIN: accumulator buffer of this unit
        const uint32_t gk0 = gk;
        for (int kb = 0; kb < nkb && ok; kb++) {   // kb counts from this unit's first k-block
          const uint32_t g = gk0 + kb;
          const int s = g % C::NST;
          ok = warp_wait(&bars->full[s], (g / C::NST) & 1, abort_flag, p.status, p.wait_ns);
          if (!ok) break;
          tc_fence_after();
          const uint32_t aA = smem_base + s * C::STAGE;
          const uint64_t adesc = sdesc_sw128(aA), bdesc = sdesc_sw128(aA + C::A_BYTES);
          if (C::HASH) {
#pragma unroll
            for (int part = 0; part < C::PARTS; part++) {
              if (part == 1 && kb * kKB + 64 >= k) break;   // k % 128 == 64 with r = 64
              const bool cstart = C::SPAN == 1 || (kb & 1) == 0;
              const bool cend = C::SPAN == 1 || (kb & 1) == 1;
#pragma unroll
              for (int a = 0; a < C::NACC; a++) {
                if (a >= nacc) break;
                if (cstart) {
                  const uint32_t w = C::MINE ? writes[a]++ : snaps[a];
                  ok = warp_wait(&bars->acc_empty[a], (w & 1) ^ 1, abort_flag, p.status, p.wait_ns);
                  if (!ok) break;
                  tc_fence_after();
                }
                // MINE: a = row half (X, Y), full 256 columns; FWD: a = column half (16-byte desc units)
                const uint64_t ad = adesc + (C::MINE ? a * (128 * kKB / 16) : 0);
                const uint64_t bd = bdesc + (C::MINE ? 0 : a * (128 * kKB / 16));
                const uint32_t dcol = tmem + a * C::ACC_N;
                if (leader) {
#pragma unroll
                  for (int ks = part * (4 / C::PARTS); ks < (part + 1) * (4 / C::PARTS); ks++)
                    mma_i8(dcol, ad + 2 * ks, bd + 2 * ks, id_acc, (kb == 0 && ks == 0) ? 0u : 1u);
                }
                if (cend) {
                  if (leader) mma_commit(&bars->acc_full[a]);
                  snaps[a]++;
                }
              }
              if (!ok) break;
            }
          } else {
#pragma unroll
            for (int a = 0; a < C::NACC; a++) {
              const int ba = MODE == MODE_PLAIN ? pbuf : a;
              if (kb == 0) {
                const uint32_t uses = MODE == MODE_PLAIN ? (uint32_t)(local >> 1) : snaps[a];
                ok = warp_wait(&bars->acc_empty[ba], (uses & 1) ^ 1, abort_flag, p.status, p.wait_ns);
                if (!ok) break;
                tc_fence_after();
              }
              const uint64_t bd = bdesc + (MODE == MODE_FWD ? a * (128 * kKB / 16) : 0);
              const uint32_t dcol = tmem + (MODE == MODE_PLAIN ? pbuf * 256 : a * 128);
              if (leader) {
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
                  mma_i8(dcol, adesc + 2 * ks, bd + 2 * ks, id_acc, (kb == 0 && ks == 0) ? 0u : 1u);
              }
              if (kb == nkb - 1) {
                if (leader) mma_commit(&bars->acc_full[ba]);
                if (MODE != MODE_PLAIN) snaps[a]++;
              }
            }
          }
          if (!ok) break;
          if (leader) mma_commit(&bars->empty[s]);
        }
        gk = gk0 + nkb;
        // ---- MINE_FWD: the correction R of each finished accumulator, into its own columns:
        // highest limb first (accumulate off), the epilogue shifts R by 7 bits before each lower
        // limb accumulates on top (Horner), c_ready after each limb
        if (FWDH && L > 0) {
          for (int li = L - 1; li >= 0 && ok; li--) {
            for (int kb = 0; kb < cblocks && ok; kb++, gk++) {
              const int s = gk % C::NST;
              ok = warp_wait(&bars->full[s], (gk / C::NST) & 1, abort_flag, p.status, p.wait_ns);
              if (!ok) break;
              tc_fence_after();
              const uint32_t aA = smem_base + s * C::STAGE;
              const uint64_t adesc = sdesc_sw128(aA), bdesc = sdesc_sw128(aA + C::A_BYTES);
              for (int a = 0; a < nacc && ok; a++) {
                if (kb == 0) {
                  if (li == L - 1)   // the last snapshot's release
                    ok = warp_wait(&bars->acc_empty[a], (writes[a]++ & 1) ^ 1, abort_flag, p.status, p.wait_ns);
                  else
                    ok = warp_wait(&bars->c_shifted[a], shifted[a]++ & 1, abort_flag, p.status, p.wait_ns);
                  if (!ok) break;
                  tc_fence_after();
                }
                if (leader) {
#pragma unroll
                  for (int ks = 0; ks < 4; ks++)
                    mma_i8(tmem + a * 256, adesc + a * (128 * kKB / 16) + 2 * ks, bdesc + 2 * ks, id_acc,
                           (li == L - 1 && kb == 0 && ks == 0) ? 0u : 1u);
                  if (kb == cblocks - 1) mma_commit(&bars->c_ready[a]);
                }
              }
              if (!ok) break;
              if (leader) mma_commit(&bars->empty[s]);
            }
          }
        }
      }
      // drain: every MMA issued by the leader has completed before TMEM is released
      if (leader) mma_commit(&bars->drain);
      warp_wait(&bars->drain, 0, abort_flag, p.status, p.wait_ns);
    }
  } else if (warp < kEpiWarps) {
    // ------------------------------------------------------------ epilogue warps
    const int q = warp & 3, cb = warp >> 2;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    // message slot of this thread's tile after the reduce-scatter: g = lane % 8, t = lane / 8
    const int tslot = (lane & 7) * 4 + (lane >> 3);
    uint32_t snaps[2] = {0, 0};
    uint32_t cready[2] = {0, 0};    // MINE_FWD: c_ready waits per accumulator
    uint32_t r_waits = 0;
    int local = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.nunits && ok; u += gridDim.x, local++) {
      int m0, n0, kb0, nkb, bt;
      unit_span(p, u, C::UM, kblocks, m0, n0, kb0, nkb, bt);
      if (MODE == MODE_PLAIN) {
        const int b = local & 1;
        ok = warp_wait(&bars->acc_full[b], (local >> 1) & 1, abort_flag, p.status, p.wait_ns);
        if (!ok) break;
        tc_fence_after();
        if (p.swiglu) {
          // gate columns 32 cb .. 32 cb + 31 and their up columns + 128: 32 outputs per row, built
          // in two halves, then stored 4 rows x 32 columns per instruction through the warp's tile
          uint32_t* const tile = tiles + warp * C::TILE_WORDS;
          const int row = m0 + 32 * q + lane, f0 = n0 / 2 + 32 * cb;
          const float sx = row < p.m ? p.a_scale[row] : 0.f;
#pragma unroll 1
          for (int hh = 0; hh < 2; hh++) {
            uint32_t g[16], u[16];
            tmem_ld_32x32b_x16(lane_base + tmem + b * 256 + 32 * cb + 16 * hh, g);
            tmem_ld_32x32b_x16(lane_base + tmem + b * 256 + 128 + 32 * cb + 16 * hh, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i++) {
              const int f = f0 + 16 * hh + i;
              float hv = 0.f;
              if (f < p.n)
                hv = det_swiglu(__fmul_rn(__fmul_rn(__int2float_rn((int)g[i]), sx), __ldg(p.b_scale + f)),
                                __fmul_rn(__fmul_rn(__int2float_rn((int)u[i]), sx), __ldg(p.b_scale + p.n + f)));
              tile[lane * 33 + 16 * hh + i] = __float_as_uint(hv);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) ACC_ARRIVE(&bars->acc_empty[b]);
          const int cl = 4 * (lane & 7), c = f0 + cl;
#pragma unroll
          for (int pass = 0; pass < 8; pass++) {
            const int rl = pass * 4 + (lane >> 3), rr = m0 + 32 * q + rl;
            const uint32_t* t = tile + rl * 33 + cl;
            if (rr < p.m && c < p.n)
              *reinterpret_cast<uint4*>(static_cast<float*>(p.out) + (uint64_t)rr * p.n + c) =
                  make_uint4(t[0], t[1], t[2], t[3]);
          }
          __syncwarp();
          continue;
        }
        const uint32_t col = tmem + b * 256 + cb * 64;
#pragma unroll 1
        for (int h = 0; h < 2; h++) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(lane_base + col + h * 32, v);
          tmem_wait_ld();
          const int row = m0 + 32 * q + lane, c0 = n0 + cb * 64 + h * 32;
          if (p.nsplit > 1) {
            // split-K partial: integer adds into the zeroed int32 product commute, so the sum is
            // exact whatever order the splits land in
            if (row < p.m && c0 < p.n) {
              int32_t* o = static_cast<int32_t*>(p.out) + (uint64_t)row * p.n + c0;
#pragma unroll
              for (int i = 0; i < 32; i++)
                if (c0 + i < p.n) atomicAdd(o + i, (int32_t)v[i]);
            }
          } else if (p.out_mode != UWC_OUT_NONE && (p.n & 3) == 0) {
            // through this warp's tile: 4 rows x 32 columns per store instruction
            uint32_t* const tile = tiles + warp * C::TILE_WORDS;
#pragma unroll
            for (int j = 0; j < 32; j++) tile[lane * 33 + j] = v[j];
            __syncwarp();
            const int cl = 4 * (lane & 7), c = c0 + cl;
#pragma unroll
            for (int pass = 0; pass < 8; pass++) {
              const int rl = pass * 4 + (lane >> 3), r = m0 + 32 * q + rl;
              const uint32_t* t = tile + rl * 33 + cl;
              if (r < p.m && c < p.n)
                store4(p, bt * p.m + r, c, (int32_t)t[0], (int32_t)t[1], (int32_t)t[2], (int32_t)t[3]);
            }
            __syncwarp();
          } else {
            store_row32(p, row, c0, reinterpret_cast<const int32_t*>(v));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) ACC_ARRIVE(&bars->acc_empty[b]);
        continue;
      }

      if (C::MINE) {
        // ---- the mining schedules: accumulators X (a = 0, rows m0..m0+127) and Y (a = 1), this
        // warp's 32 rows (quadrant q) x 64 columns (block cb) of each
        const bool hasY = m0 + 128 < p.m;
        const uint32_t colX = tmem + lane_base + cb * 64;
        const int rb = q >> 1;   // 64-row half of the 128-row accumulator, for the message slot
        const int slot[2] = {((0 * 2 + rb) * 4 + cb) * 32 + tslot, ((1 * 2 + rb) * 4 + cb) * 32 + tslot};
        const int c0 = n0 + cb * 64;
        auto row_of = [&](int a) { return m0 + a * 128 + 32 * q + lane; };
        // this thread's raw product slots for accumulator a in the CTA's staging block
        auto stage_of = [&](int a) {
          return reinterpret_cast<uint4*>(p.stage + ((uint64_t)blockIdx.x * 2 + a) * (kStageWords / 2));
        };
        // consume one snapshot of accumulator a: read 64 values, release the accumulator, fold
        auto consume = [&](int a, bool last) -> uint32_t {
          ok = warp_wait(&bars->acc_full[a], snaps[a] & 1, abort_flag, p.status, p.wait_ns);
          if (!ok) return 0u;
          snaps[a]++;
          tc_fence_after();
          uint32_t v[32], v2[32];
          tmem_ld_32x32b_x32(colX + a * 256, v);
          tmem_ld_32x32b_x32(colX + a * 256 + 32, v2);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) ACC_ARRIVE(&bars->acc_empty[a]);
          uint32_t pt[4] = {0u, 0u, 0u, 0u};
          fold_row32(v, pt);
          fold_row32(v2, pt);
          // the last snapshot of a forward: the raw values wait in the staging block until the
          // unit's hashes are done (and the correction has landed), then go out
          if (FWDH && last) store_raw64(stage_of(a), threadIdx.x, v, v2);
          return reduce_scatter4(pt, lane);
        };
        // the previous unit's tile hashes clear the message words this unit reduces into
        bool clear_pending = local > 0;
        auto chunk = [&](int c, bool last) {
          const int sl = c & 15;
          // slot sl is updated again by chunks c + 16, c + 32, ... < nch: the contribution of
          // chunk c is rotated 13 bits for each of those later updates
          const int rot = (13 * ((nch - 1 - c) >> 4)) & 31;
#pragma unroll
          for (int a = 0; a < 2; a++) {
            if (a == 1 && !hasY) break;
            const uint32_t x = consume(a, last);
            if (!ok) break;
            if (clear_pending) {
              // the message words are zero again: hashes done (MINE), transpose tiles re-zeroed (FWD)
              ok = warp_wait(FWDH ? &bars->tiles_done : &bars->hash_done, (local - 1) & 1, abort_flag, p.status,
                             p.wait_ns);
              clear_pending = false;
              if (!ok) break;
            }
            red_xor_shared(msg + sl * kMaxTiles + slot[a], __funnelshift_l(x, x, rot));
          }
        };
        // the last chunk of a forward (which also writes the output) is peeled off the loop; two
        // chunks per iteration let the scheduler interleave one chunk's fold with the next's loads
        // (C3 r = 64: 0.6195 -> 0.6072 ms)
#pragma unroll 2
        for (int c = 0; c < (FWDH ? nch - 1 : nch) && ok; c++) chunk(c, false);
        if (FWDH && ok) chunk(nch - 1, true);
        if (!ok) break;
        // every thread's reductions of this unit are in shared memory: each thread hashes one tile
        mbar_arrive(&bars->hash_ready);
        ok = warp_wait(&bars->hash_ready, local & 1, abort_flag, p.status, p.wait_ns);
        if (!ok) break;
        hash_tile(p, msg, m0, n0, threadIdx.x);
        mbar_arrive(&bars->hash_done);   // waited on before the next unit's first reduction (MINE)
        if (FWDH) {
          // ---- the output: correction (Horner: shift R by 7 bits between limbs), then out = raw - R,
          // scaled. The message buffer is idle until the next unit's first reduction: each warp
          // transposes its rows through 2 KiB of it, so the stores are row-contiguous.
          for (int step = 0; step + 1 < L && ok; step++) {
#pragma unroll
            for (int a = 0; a < 2; a++) {
              if ((a == 1 && !hasY) || !ok) break;
              ok = warp_wait(&bars->c_ready[a], cready[a]++ & 1, abort_flag, p.status, p.wait_ns);
              if (!ok) break;
              tc_fence_after();
#pragma unroll 1
              for (int hh = 0; hh < 2; hh++) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(colX + a * 256 + hh * 32, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] <<= 7;
                tmem_st_32x32b_x32(colX + a * 256 + hh * 32, v);
              }
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) ACC_ARRIVE(&bars->c_shifted[a]);
            }
          }
          if (!ok) break;
          // every thread has read and cleared its tile's message words
          ok = warp_wait(&bars->hash_done, local & 1, abort_flag, p.status, p.wait_ns);
          if (!ok) break;
          uint4* const tile = reinterpret_cast<uint4*>(msg) + warp * 128;   // 32 rows x 16 words
#pragma unroll
          for (int a = 0; a < 2; a++) {
            if ((a == 1 && !hasY) || !ok) break;
            if (L > 0) {
              ok = warp_wait(&bars->c_ready[a], cready[a]++ & 1, abort_flag, p.status, p.wait_ns);
              if (!ok) break;
              tc_fence_after();
            }
            const uint4* st = stage_of(a);
#pragma unroll 1
            for (int sl = 0; sl < 4; sl++) {   // 16-column slices of the warp's 64 columns
              uint32_t w[16];
#pragma unroll
              for (int i = 0; i < 4; i++) {
                const uint4 t = __ldcg(st + (4 * sl + i) * 512 + threadIdx.x);
                w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
              }
              if (L > 0) {
                uint32_t rr[16];
                tmem_ld_32x32b_x16(colX + a * 256 + 16 * sl, rr);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; i++) w[i] -= rr[i];
              }
              const int nq = convert16(p, row_of(a), c0 + 16 * sl, w);
              // row `lane` of the tile, quads swizzled by (row >> 1) & 3: conflict-free both ways
#pragma unroll
              for (int i = 0; i < 4; i++)
                if (i < nq) tile[lane * 4 + (i ^ ((lane >> 1) & 3))] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
              __syncwarp();
              if (c0 < p.n) {
                // nq lanes per row, 32 / nq rows per instruction, 16 contiguous bytes per lane
                const int per = 32 / nq;
#pragma unroll 1
                for (int r0 = 0; r0 < 32; r0 += per) {
                  const int tr = r0 + lane / nq, qd = lane % nq, row = m0 + a * 128 + 32 * q + tr;
                  const uint4 val = tile[tr * 4 + (qd ^ ((tr >> 1) & 3))];
                  if (row < p.m) {
                    uint8_t* o = static_cast<uint8_t*>(p.out) +
                                 ((uint64_t)row * p.n + c0 + 16 * sl) * (p.out_mode == UWC_OUT_BF16 ? 2 : 4);
                    reinterpret_cast<uint4*>(o)[qd] = val;
                  }
                }
              }
              __syncwarp();
            }
            if (L > 0) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) ACC_ARRIVE(&bars->acc_empty[a]);   // the accumulator is free for the next unit
            }
          }
          if (!ok) break;
          // the tile goes back to zero (message words of the next unit), then the hand-off
#pragma unroll
          for (int i = 0; i < 4; i++) tile[lane * 4 + i] = make_uint4(0u, 0u, 0u, 0u);
          mbar_arrive(&bars->tiles_done);
        }
        continue;
      }

      // ---- FWD (a = cb / 2, the column half; this warp's columns (cb % 2) * 64) and CORR
      const int a0 = cb >> 1;
      const uint32_t col0 = tmem + lane_base + a0 * 128 + (cb & 1) * 64;

      if (C::CORR && !(MODE == MODE_CORR && L <= 2)) {
        // Horner: R <<= 7 between limbs (all 16 warps, 64 columns of R each)
        for (int step = 0; step + 1 < L && ok; step++) {
          ok = warp_wait(&bars->r_full, r_waits++ & 1, abort_flag, p.status, p.wait_ns);
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int hh = 0; hh < 2; hh++) {
            uint32_t v[32];
            const uint32_t ta = tmem + 256 + cb * 64 + hh * 32 + lane_base;
            tmem_ld_32x32b_x32(ta, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] <<= 7;
            tmem_st_32x32b_x32(ta, v);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) ACC_ARRIVE(&bars->r_scaled);
        }
        if (!ok) break;
      }
      if (MODE == MODE_CORR) {
        // out = acc - R (R = 0 without denoising), acc read back from the summed int32 product,
        // then scaled / converted to the output format
        if (L > 0) {
          ok = warp_wait(&bars->r_full, r_waits++ & 1, abort_flag, p.status, p.wait_ns);
          if (!ok) break;
          tc_fence_after();
        }
        uint32_t* const tile = tiles + warp * C::TILE_WORDS;
#pragma unroll 1
        for (int hh = 0; hh < 2; hh++) {
          const int c0 = n0 + cb * 64 + hh * 32;
          // R for this warp's 32 rows x 32 columns (thread = row), staged transposed in shared memory
          uint32_t rr[32];
          if (L > 2) {
            tmem_ld_32x32b_x32(tmem + 256 + cb * 64 + hh * 32 + lane_base, rr);
            tmem_wait_ld();
          } else if (L > 0) {
            // R = P0 + (P1 << 7): the same int32 value as the Horner form
            const uint32_t ta = tmem + cb * 64 + hh * 32 + lane_base;
            tmem_ld_32x32b_x32(ta, rr);
            if (L == 2) {
              uint32_t r1[32];
              tmem_ld_32x32b_x32(ta + 256, r1);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; i++) rr[i] += r1[i] << 7;
            } else {
              tmem_wait_ld();
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i++) rr[i] = 0u;
          }
#pragma unroll
          for (int j = 0; j < 32; j++) tile[lane * 33 + j] = rr[j];
          __syncwarp();
          // 4 rows x 32 columns per pass: 8 lanes per row, 4 consecutive columns per lane; all eight
          // passes' loads are issued before the first use (4 KiB in flight per warp)
          const int cl = 4 * (lane & 7), c = c0 + cl;
          int4 a[8];
#pragma unroll
          for (int pass = 0; pass < 8; pass++) {
            const int row = m0 + 32 * q + pass * 4 + (lane >> 3);
            a[pass] = (row < p.m && c < p.n) ? __ldcs(reinterpret_cast<const int4*>(p.acc_in + (uint64_t)row * p.n + c))
                                             : make_int4(0, 0, 0, 0);
          }
#pragma unroll
          for (int pass = 0; pass < 8; pass++) {
            const int rl = pass * 4 + (lane >> 3), row = m0 + 32 * q + rl;
            if (row < p.m && c < p.n) {
              const uint32_t* t = tile + rl * 33 + cl;
              store4(p, row, c, a[pass].x - (int32_t)t[0], a[pass].y - (int32_t)t[1], a[pass].z - (int32_t)t[2],
                     a[pass].w - (int32_t)t[3]);
            }
          }
          __syncwarp();
        }
        if (L > 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) ACC_ARRIVE(&bars->r_empty);
        }
        continue;
      }

      // FWD: the unit's only snapshot: out = acc - R for this warp's 32 rows x 64 columns
      ok = warp_wait(&bars->acc_full[a0], snaps[a0] & 1, abort_flag, p.status, p.wait_ns);
      if (!ok) break;
      snaps[a0]++;
      tc_fence_after();
      if (L > 0) {
        ok = warp_wait(&bars->r_full, r_waits++ & 1, abort_flag, p.status, p.wait_ns);
        if (!ok) break;
        tc_fence_after();
      }
      if (p.out_mode != UWC_OUT_NONE) {
#pragma unroll 1
        for (int hh = 0; hh < 2; hh++) {
          uint32_t w[32];
          tmem_ld_32x32b_x32(col0 + hh * 32, w);
          tmem_wait_ld();
          if (L > 0) {
#pragma unroll
            for (int qq = 0; qq < 2; qq++) {
              uint32_t rr[16];
              tmem_ld_32x32b_x16(tmem + 256 + cb * 64 + hh * 32 + qq * 16 + lane_base, rr);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; i++) w[qq * 16 + i] -= rr[i];
            }
          }
          store_row32(p, m0 + 32 * q + lane, n0 + cb * 64 + hh * 32, reinterpret_cast<const int32_t*>(w));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        ACC_ARRIVE(&bars->acc_empty[a0]);
        if (L > 0) ACC_ARRIVE(&bars->r_empty);
      }
    }
  }

  // ------------------------------------------------------------ teardown
  if (*abort_flag) {
    // let in-flight TMA copies and MMAs land before the CTA (and its shared memory) goes away
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 20000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
}

// Test hooks (uwc_test_hook): the bound of every wait, and whether launches withhold their copies.
std::atomic<uint64_t> g_wait_ns{0};
std::atomic<int> g_withhold{0};

template <int MODE, int R>
int launch(Params p, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& ca, const CUtensorMap& cb,
           cudaStream_t st) {
  const uint64_t ns = g_wait_ns.load();
  p.wait_ns = ns ? ns : UWC_WAIT_TIMEOUT_NS;
  p.withhold = g_withhold.load();
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(k_noisy_gemm<MODE, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<MODE, R>::SMEM) != cudaSuccess) {
      cudaGetLastError();
      return UWC_ERR_CUDA;
    }
    configured[dev] = 1;
  }
  const int grid = std::min(p.nunits, uwc_num_sms());
  k_noisy_gemm<MODE, R><<<grid, kThreads, Cfg<MODE, R>::SMEM, st>>>(a, b, ca, cb, p);
  uwc_count_launch();
  return uwc_launch_status();
}

template <int MODE>
int launch_r(const Params& p, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& ca,
             const CUtensorMap& cb, cudaStream_t st) {
  if (p.r == 64) return launch<MODE, 64>(p, a, b, ca, cb, st);
  if (p.r == 128) return launch<MODE, 128>(p, a, b, ca, cb, st);
  return launch<MODE, 256>(p, a, b, ca, cb, st);
}

}  // namespace

namespace {
// Workspace of a hashed call with an output: per CTA one staging block of kStageWords int32 (a unit's
// raw products wait there, thread-interleaved, for the unit's hashes and correction; 256 KiB).
uint64_t stage_bytes(int flags, int out_mode) {
  const bool staged = (flags & UWC_FLAG_HASH) && out_mode != UWC_OUT_NONE;
  return staged ? (uint64_t)uwc_num_sms() * kStageWords * 4 : 0;
}
// Skinny plain GEMMs (decode-sized m, tensor-parallel shards of n) have fewer 128 x 256 output
// blocks than half the SMs: they split k across units and add int32 partials.
bool split_k(int m, int n) {
  const int blocks = ((m + 127) / 128) * ((n + kUN - 1) / kUN);
  return 2 * blocks <= uwc_num_sms();
}
}  // namespace

uint64_t uwc_wait_ns() { return g_wait_ns.load(); }

extern "C" int uwc_test_hook(int hook, long long value) {
  if (hook == UWC_HOOK_WAIT_NS && value >= 0) {
    g_wait_ns.store((uint64_t)value);
    uwc_stream_set_wait_ns((uint64_t)value);
    return UWC_OK;
  }
  if (hook == UWC_HOOK_TP_TWO_PHASE && value >= 1 && value <= 9) {
    uwc_tp_set_two_phase_min((int)value);
    return UWC_OK;
  }
  if (hook == UWC_HOOK_STREAM_PDL && (value == 0 || value == 1)) {
    uwc_stream_set_pdl((int)value);
    uwc_row_set_pdl((int)value);
    return UWC_OK;
  }
  if (hook == UWC_HOOK_WITHHOLD && (value == 0 || value == 1)) {
    g_withhold.store((int)value);
    return UWC_OK;
  }
  return UWC_ERR_ARG;
}

extern "C" uint64_t uwc_gemm_workspace_bytes(int m, int n, int flags, int out_mode) {
  uint64_t bytes = stage_bytes(flags, out_mode);
  if (!flags && m <= 64) return bytes;   // the weight-streaming GEMM: no workspace
  // split-K with a scaled output: the int32 product is summed here, then scaled by a second pass
  if (!flags && (out_mode == UWC_OUT_F32 || out_mode == UWC_OUT_BF16) && m > 0 && n > 0 && split_k(m, n))
    bytes += (uint64_t)m * n * 4;
  return bytes;
}

namespace {
// uwc_gemm, plus the fused output steps of uwc_gemm_epi for plain calls: resid (F32 out + x) and
// swiglu (B = [gate; up] with 2n rows, F32 out m x n).
int gemm_impl(const int8_t* A, const int8_t* B, int m, int n, int k, int r, int flags, const int8_t* corrA,
              const int8_t* corrB, const int32_t* maxabs, int lmax, const uint32_t* key, const uint32_t* target,
              uint32_t* wins, int max_wins, const float* a_scale, const float* b_scale, void* out, int out_mode,
              void* workspace, uint64_t workspace_bytes, void* stream, const float* resid, int swiglu) {
  const bool hash = flags & UWC_FLAG_HASH, denoise = flags & UWC_FLAG_DENOISE;
  if (!A || !B || (flags & ~3) || out_mode < 0 || out_mode > 3) return UWC_ERR_ARG;
  if (out_mode != UWC_OUT_NONE && !out) return UWC_ERR_ARG;
  if ((out_mode == UWC_OUT_BF16 || out_mode == UWC_OUT_F32) && (!a_scale || !b_scale)) return UWC_ERR_ARG;
  if (hash && (!key || !target || !wins || max_wins < 0)) return UWC_ERR_ARG;
  if (denoise && (!corrA || !corrB || !maxabs || lmax < 1 || lmax > 4)) return UWC_ERR_ARG;
  if (m <= 0 || n <= 0 || k <= 0 || k % 16) return UWC_ERR_SHAPE;
  if (hash || denoise) {
    if (m % 64 || n % 64 || k % 64) return UWC_ERR_SHAPE;
    if (r != 64 && r != 128 && r != 256) return UWC_ERR_SHAPE;
    if (k % r) return UWC_ERR_SHAPE;
  }
  if (out_mode == UWC_OUT_BF16 ? (n % 8) : (out_mode != UWC_OUT_NONE && n % 4)) return UWC_ERR_SHAPE;
  if ((((uintptr_t)A) | ((uintptr_t)B) | ((uintptr_t)out) | ((uintptr_t)corrA) | ((uintptr_t)corrB) |
       ((uintptr_t)workspace)) & 15)
    return UWC_ERR_ALIGN;
  UWC_CHECK_DEVICE();
  const uint64_t need = swiglu ? 0 : uwc_gemm_workspace_bytes(m, n, flags, out_mode);
  if (need && (!workspace || workspace_bytes < need)) return UWC_ERR_SCRATCH;
  // decode-sized m: W streamed once, k split over a cluster, the output step in its epilogue
  if (!hash && !denoise && !resid && !swiglu && out_mode != UWC_OUT_NONE && uwc_stream_gemm_fits(m, n, k)) {
    const int epi = out_mode == UWC_OUT_I32 ? UWC_SEPI_I32 : (out_mode == UWC_OUT_F32 ? UWC_SEPI_F32 : UWC_SEPI_BF16);
    return uwc_gemm_stream(A, B, m, n, k, a_scale, b_scale, nullptr, out, epi, stream);
  }

  Params p{};
  p.m = m; p.n = n; p.k = k; p.r = r;
  p.hash = hash; p.denoise = denoise; p.lmax = lmax; p.out_mode = out_mode; p.max_wins = max_wins;
  p.maxabs = maxabs; p.key = key; p.target = target; p.wins = wins;
  p.a_scale = a_scale; p.b_scale = b_scale; p.out = out;
  p.resid = resid; p.swiglu = swiglu;
  p.status = uwc_status_ptr();
  p.one = 1u;
  p.b_bdiv = 1;
  p.nn = (n + kUN - 1) / kUN;
  cudaStream_t st = (cudaStream_t)stream;

  CUtensorMap ta, tb, tca, tcb;
  // A-side boxes: 256 rows for the mining schedule, 128 otherwise
  const int UM = hash ? 256 : 128;
  int rc = uwc_make_tmap_2d(&ta, A, (uint64_t)m, (uint64_t)k, (uint64_t)k, UM, kKB);
  if (rc == UWC_OK) rc = uwc_make_tmap_2d(&tb, B, (uint64_t)n, (uint64_t)k, (uint64_t)k, kUN, kKB);
  if (rc != UWC_OK) return rc;
  if (denoise) {
    rc = uwc_make_tmap_2d(&tca, corrA, (uint64_t)lmax * m, (uint64_t)2 * r, (uint64_t)2 * r, UM, kKB);
    if (rc == UWC_OK) rc = uwc_make_tmap_2d(&tcb, corrB, (uint64_t)lmax * n, (uint64_t)2 * r, (uint64_t)2 * r, kUN, kKB);
    if (rc != UWC_OK) return rc;
  } else {
    tca = ta;
    tcb = tb;
  }

  const int kblocks = (k + kKB - 1) / kKB;
  p.nsplit = 1;
  p.kps = kblocks;
  if (!hash) {
    p.nm = (m + 127) / 128;
    p.nunits = p.nm * p.nn;
    if (denoise) return launch<MODE_FWD, 0>(p, ta, tb, tca, tcb, st);
    if (swiglu) {
      // units of 128 outputs: 128 gate rows of B over their 128 up rows (two 128-row boxes)
      rc = uwc_make_tmap_2d(&tcb, B, (uint64_t)2 * n, (uint64_t)k, (uint64_t)k, 128, kKB);
      if (rc != UWC_OK) return rc;
      p.nn = (n + 127) / 128;
      p.nunits = p.nm * p.nn;
      return launch<MODE_PLAIN, 0>(p, ta, tb, tca, tcb, st);
    }
    if (out_mode == UWC_OUT_NONE || !split_k(m, n) || kblocks < 2)
      return launch<MODE_PLAIN, 0>(p, ta, tb, tca, tcb, st);
    // split-K: each unit owns a k-block range of one output block and adds its int32 partial into
    // the zeroed product (`out` itself for I32, else the workspace, scaled by a second pass)
    const int splits = std::min(kblocks, std::max(1, uwc_num_sms() / p.nunits));
    p.kps = (kblocks + splits - 1) / splits;
    p.nsplit = (kblocks + p.kps - 1) / p.kps;
    int32_t* acc = out_mode == UWC_OUT_I32 ? static_cast<int32_t*>(out) : static_cast<int32_t*>(workspace);
    if (cudaMemsetAsync(acc, 0, (size_t)m * n * 4, st) != cudaSuccess) {
      cudaGetLastError();
      return UWC_ERR_CUDA;
    }
    p.out = acc;
    p.out_mode = UWC_OUT_I32;
    p.nunits *= p.nsplit;
    rc = launch<MODE_PLAIN, 0>(p, ta, tb, tca, tcb, st);
    if (rc != UWC_OK || out_mode == UWC_OUT_I32) return rc;
    Params q = p;
    q.nsplit = 1;
    q.kps = kblocks;
    q.nunits = q.nm * q.nn;
    q.out = out;
    q.out_mode = out_mode;
    q.acc_in = acc;
    return launch<MODE_CORR, 0>(q, ta, tb, tca, tcb, st);
  }

  // Hashed: the mining schedule hashes every tile; with an output the same kernel writes it (and
  // subtracts the correction first when denoising)
  p.nm = (m + 255) / 256;
  p.nunits = p.nm * p.nn;
  if (out_mode == UWC_OUT_NONE) {
    p.denoise = 0;
    return launch_r<MODE_MINE>(p, ta, tb, tca, tcb, st);
  }
  p.stage = stage_bytes(flags, out_mode) ? static_cast<int32_t*>(workspace) : nullptr;
  return launch_r<MODE_MINE_FWD>(p, ta, tb, tca, tcb, st);
}
}  // namespace

extern "C" int uwc_gemm(const int8_t* A, const int8_t* B, int m, int n, int k, int r, int flags, const int8_t* corrA,
                        const int8_t* corrB, const int32_t* maxabs, int lmax, const uint32_t* key,
                        const uint32_t* target, uint32_t* wins, int max_wins, const float* a_scale,
                        const float* b_scale, void* out, int out_mode, void* workspace, uint64_t workspace_bytes,
                        void* stream) {
  return gemm_impl(A, B, m, n, k, r, flags, corrA, corrB, maxabs, lmax, key, target, wins, max_wins, a_scale,
                   b_scale, out, out_mode, workspace, workspace_bytes, stream, nullptr, 0);
}

namespace {
int epi_out_mode(int epi) {
  switch (epi) {
    case UWC_SEPI_I32: return UWC_OUT_I32;
    case UWC_SEPI_BF16: return UWC_OUT_BF16;
    default: return UWC_OUT_F32;
  }
}
}  // namespace

extern "C" uint64_t uwc_gemm_epi_workspace_bytes(int m, int n, int epi) {
  epi &= ~UWC_SEPI_EARLY_W;
  if (m <= 0 || n <= 0 || epi < UWC_SEPI_I32 || epi > UWC_SEPI_SWIGLU) return 0;
  if (m <= 64 || epi == UWC_SEPI_SWIGLU) return 0;
  return uwc_gemm_workspace_bytes(m, n, 0, epi_out_mode(epi));
}

extern "C" int uwc_gemm_epi(const int8_t* A, const int8_t* W, int m, int n, int k, const float* a_scale,
                            const float* w_scale, const float* resid, void* out, int epi, void* workspace,
                            uint64_t workspace_bytes, void* stream) {
  const int kind = epi & ~UWC_SEPI_EARLY_W;
  if (kind < UWC_SEPI_I32 || kind > UWC_SEPI_SWIGLU) return UWC_ERR_ARG;
  if (resid && kind != UWC_SEPI_RESID) return UWC_ERR_ARG;
  // decode-sized m: the weight-streaming GEMM (its own argument checks)
  if (uwc_stream_gemm_fits(m, n, k) && (kind != UWC_SEPI_SWIGLU || n % 128 == 0))
    return uwc_gemm_stream(A, W, m, n, k, a_scale, w_scale, resid, out, epi, stream);
  if (kind == UWC_SEPI_SWIGLU) {
    if (n % 8) return UWC_ERR_SHAPE;   // n / 2 outputs per row, 16-byte rows
    return gemm_impl(A, W, m, n / 2, k, 0, 0, nullptr, nullptr, nullptr, 0, nullptr, nullptr, nullptr, 0, a_scale,
                     w_scale, out, UWC_OUT_F32, workspace, workspace_bytes, stream, nullptr, 1);
  }
  return gemm_impl(A, W, m, n, k, 0, 0, nullptr, nullptr, nullptr, 0, nullptr, nullptr, nullptr, 0, a_scale, w_scale,
                   out, epi_out_mode(kind), workspace, workspace_bytes, stream, kind == UWC_SEPI_RESID ? resid : nullptr,
                   0);
}

// Batched exact int8 GEMM, int32 out: out[bt] (m x n) = A[bt] B[bt / b_bdiv]^T for bt < nbatch, A[bt]
// the m x k rows from row bt * a_brows, B[g] the n x k rows from row g * b_brows (both k-contiguous
// row-major with row length k). causal: 0 all blocks; 1 skip 128 x 256 blocks no row sees (row t
// sees columns j <= cshift + t); 2 stop each row block's k range after key cshift + (m0 % qrows) + 127
// (A = [P_hi; P_lo] of qrows rows each). The attention's Q K^T (causal 1) and P V (causal 2).
extern "C" int uwc_gemm_batched(const int8_t* A, const int8_t* B, int m, int n, int k, int nbatch, long long a_brows,
                                long long b_brows, int b_bdiv, int causal, int cshift, int qrows, int32_t* out,
                                void* stream) {
  if (!A || !B || !out || nbatch <= 0 || b_bdiv <= 0 || causal < 0 || causal > 2 || cshift < 0) return UWC_ERR_ARG;
  if (m <= 0 || n <= 0 || k <= 0 || k % 16 || n % 4 || a_brows < m || b_brows < n) return UWC_ERR_SHAPE;
  if (causal == 2 && (qrows <= 0 || qrows % 128 || m % qrows)) return UWC_ERR_SHAPE;
  if ((((uintptr_t)A) | ((uintptr_t)B) | ((uintptr_t)out)) & 15) return UWC_ERR_ALIGN;
  const long long arows = (long long)(nbatch - 1) * a_brows + m, brows = (long long)((nbatch - 1) / b_bdiv) * b_brows + n;
  if (arows > 0x7fffffffLL || brows > 0x7fffffffLL) return UWC_ERR_SHAPE;
  UWC_CHECK_DEVICE();
  Params p{};
  p.m = m; p.n = n; p.k = k; p.r = 0;
  p.out_mode = UWC_OUT_I32; p.out = out;
  p.status = uwc_status_ptr();
  p.one = 1u;
  p.nsplit = 1;
  p.kps = (k + kKB - 1) / kKB;
  p.nm = (m + 127) / 128;
  p.nn = (n + kUN - 1) / kUN;
  p.nbatch = nbatch; p.a_brows = a_brows; p.b_brows = b_brows; p.b_bdiv = b_bdiv;
  p.causal = causal; p.cshift = cshift; p.qrows = qrows;
  int per = p.nm * p.nn;
  if (causal == 1) {
    per = 0;
    for (int mb = 0; mb < p.nm; mb++) per += std::min(p.nn, (cshift + mb * 128 + 128 + kUN - 1) / kUN);
  }
  p.units_per_batch = per;
  if ((long long)per * nbatch > 0x7fffffffLL) return UWC_ERR_SHAPE;
  p.nunits = per * nbatch;
  CUtensorMap ta, tb;
  int rc = uwc_make_tmap_2d(&ta, A, (uint64_t)arows, (uint64_t)k, (uint64_t)k, 128, kKB);
  if (rc == UWC_OK) rc = uwc_make_tmap_2d(&tb, B, (uint64_t)brows, (uint64_t)k, (uint64_t)k, kUN, kKB);
  if (rc != UWC_OK) return rc;
  return launch<MODE_PLAIN, 0>(p, ta, tb, ta, tb, (cudaStream_t)stream);
}
