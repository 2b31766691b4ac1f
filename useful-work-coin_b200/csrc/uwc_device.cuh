// Device helpers shared by the sm_100a kernels: BLAKE3 compression, mbarriers with bounded
// waits, TMA tile loads, tcgen05 (TMEM alloc / MMA / commit / ld / st) wrappers.
//
// Every wait that depends on another agent (TMA, tensor core, another warp) gives up after
// UWC_WAIT_TIMEOUT_NS of wall time, records UWC_DEV_TIMEOUT in the device status word and tells
// the caller to unwind, so a protocol bug surfaces as an error code on the host instead of a
// hung GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/uwc_b200.h"

#define UWC_DEVI __device__ __forceinline__

#ifndef UWC_WAIT_TIMEOUT_NS
#define UWC_WAIT_TIMEOUT_NS 1000000000ull  // 1 s
#endif


// ------------------------------------------------------------------ BLAKE3 (published spec)
namespace b3 {
constexpr uint32_t CHUNK_START = 1, CHUNK_END = 2, PARENT = 4, ROOT = 8, KEYED = 16;
__device__ __constant__ static const uint32_t IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                                                       0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};

UWC_DEVI uint32_t ror(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

#define UWC_B3_G(a, b, c, d, x, y)    \
  a = a + b + (x);                     \
  d = ror(d ^ a, 16);                  \
  c = c + d;                           \
  b = ror(b ^ c, 12);                  \
  a = a + b + (y);                     \
  d = ror(d ^ a, 8);                   \
  c = c + d;                           \
  b = ror(b ^ c, 7);

// a + b as an integer multiply-add by `one` (a run-time 1 the compiler cannot fold): the sum
// runs on the FMA pipe instead of the integer ALU pipe.
UWC_DEVI uint32_t add_fma(uint32_t a, uint32_t b, uint32_t one) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(one), "r"(b));
  return d;
}

// G with its additions on the FMA pipe (same values as UWC_B3_G).
#define UWC_B3_G_FMA(a, b, c, d, x, y)          \
  a = add_fma(add_fma(a, b, one), (x), one);    \
  d = ror(d ^ a, 16);                           \
  c = add_fma(c, d, one);                       \
  b = ror(b ^ c, 12);                           \
  a = add_fma(add_fma(a, b, one), (y), one);    \
  d = ror(d ^ a, 8);                            \
  c = add_fma(c, d, one);                       \
  b = ror(b ^ c, 7);

// One round on the 16-word state with message words in the current (permuted) order, then
// the spec's message permutation [2,6,3,10,7,0,4,13,1,11,12,5,9,14,15,8] applied in place.
// FMA_ADDS: additions on the FMA pipe (`one` must be 1), for kernels whose ALU pipe is busy.
template <bool FMA_ADDS = false>
UWC_DEVI void round_and_permute(uint32_t* v, uint32_t* m, uint32_t one = 1u) {
  if (FMA_ADDS) {
    UWC_B3_G_FMA(v[0], v[4], v[8], v[12], m[0], m[1]);
    UWC_B3_G_FMA(v[1], v[5], v[9], v[13], m[2], m[3]);
    UWC_B3_G_FMA(v[2], v[6], v[10], v[14], m[4], m[5]);
    UWC_B3_G_FMA(v[3], v[7], v[11], v[15], m[6], m[7]);
    UWC_B3_G_FMA(v[0], v[5], v[10], v[15], m[8], m[9]);
    UWC_B3_G_FMA(v[1], v[6], v[11], v[12], m[10], m[11]);
    UWC_B3_G_FMA(v[2], v[7], v[8], v[13], m[12], m[13]);
    UWC_B3_G_FMA(v[3], v[4], v[9], v[14], m[14], m[15]);
  } else {
    UWC_B3_G(v[0], v[4], v[8], v[12], m[0], m[1]);
    UWC_B3_G(v[1], v[5], v[9], v[13], m[2], m[3]);
    UWC_B3_G(v[2], v[6], v[10], v[14], m[4], m[5]);
    UWC_B3_G(v[3], v[7], v[11], v[15], m[6], m[7]);
    UWC_B3_G(v[0], v[5], v[10], v[15], m[8], m[9]);
    UWC_B3_G(v[1], v[6], v[11], v[12], m[10], m[11]);
    UWC_B3_G(v[2], v[7], v[8], v[13], m[12], m[13]);
    UWC_B3_G(v[3], v[4], v[9], v[14], m[14], m[15]);
  }
  uint32_t t0 = m[0], t1 = m[1], t3 = m[3], t4 = m[4], t5 = m[5], t8 = m[8], t9 = m[9], t10 = m[10], t11 = m[11],
           t12 = m[12], t13 = m[13], t14 = m[14], t15 = m[15], t6 = m[6], t7 = m[7], t2 = m[2];
  m[0] = t2; m[1] = t6; m[2] = t3; m[3] = t10; m[4] = t7; m[5] = t0; m[6] = t4; m[7] = t13;
  m[8] = t1; m[9] = t11; m[10] = t12; m[11] = t5; m[12] = t9; m[13] = t14; m[14] = t15; m[15] = t8;
}

// out = first 8 words of compress(cv, msg, counter, blen, flags). `msg` is clobbered.
template <bool FMA_ADDS = false>
UWC_DEVI void compress(const uint32_t* cv, uint32_t* msg, uint64_t counter, uint32_t blen, uint32_t flags,
                       uint32_t* out, uint32_t one = 1u) {
  uint32_t v[16];
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = cv[i];
  v[8] = IV[0]; v[9] = IV[1]; v[10] = IV[2]; v[11] = IV[3];
  v[12] = (uint32_t)counter; v[13] = (uint32_t)(counter >> 32); v[14] = blen; v[15] = flags;
#pragma unroll
  for (int r = 0; r < 7; r++) round_and_permute<FMA_ADDS>(v, msg, one);
#pragma unroll
  for (int i = 0; i < 8; i++) out[i] = v[i] ^ v[i + 8];
}

// Single-block (64-byte) hash, keyed when key != nullptr. `msg` is clobbered.
template <bool FMA_ADDS = false>
UWC_DEVI void hash64(const uint32_t* key, uint32_t* msg, uint32_t* out, uint32_t one = 1u) {
  uint32_t cv[8];
  uint32_t fl = CHUNK_START | CHUNK_END | ROOT;
  if (key) {
#pragma unroll
    for (int i = 0; i < 8; i++) cv[i] = key[i];
    fl |= KEYED;
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) cv[i] = IV[i];
  }
  compress<FMA_ADDS>(cv, msg, 0, 64, fl, out, one);
}
}  // namespace b3

// ------------------------------------------------------------------ generic helpers
UWC_DEVI uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

UWC_DEVI uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Sticky error bits go to the library's device status word, whose address the host passes in.
UWC_DEVI void set_status(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

// ------------------------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialization may start before the previous kernel of
// its stream has finished, once every CTA of that kernel has called pdl_trigger() (or exited).
// pdl_wait() blocks until the previous kernel has completed and its writes are visible; without a
// programmatic dependency both are no-ops.
UWC_DEVI void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
UWC_DEVI void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ mbarrier
UWC_DEVI void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
UWC_DEVI void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
UWC_DEVI void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Arrive without release semantics: for hand-offs that only order tensor-memory accesses (a TMEM
// read finished with tcgen05.wait::ld, then tcgen05.fence::before_thread_sync) and must not wait
// for this thread's earlier global or shared-memory writes to complete, as a release would.
UWC_DEVI void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
UWC_DEVI void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
UWC_DEVI bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false (and raises the CTA's abort
// flag and the device status) after timeout_ns (default UWC_WAIT_TIMEOUT_NS), or as soon as another
// thread of the CTA has raised the abort flag.
UWC_DEVI bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint32_t* status,
                        uint64_t timeout_ns = UWC_WAIT_TIMEOUT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > timeout_ns) {
        *abort_flag = 1;
        set_status(status, UWC_DEV_TIMEOUT);
        return false;
      }
    }
  }
}

// True in exactly one lane of the converged warp (elect.sync): the warp keeps running a role's
// schedule together, so its loop state stays warp-uniform, and only the elected lane issues.
UWC_DEVI bool elect_one() {
  uint32_t is_leader;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(is_leader));
  return is_leader != 0;
}

UWC_DEVI void named_bar_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }
UWC_DEVI void named_bar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------------ TMA
// 2D tiled load into shared memory, completion counted on `bar` (bytes). x is the innermost
// coordinate (bytes for int8 data) and must be a multiple of 16; callers only pass multiples of 128.
UWC_DEVI void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
UWC_DEVI void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------------ tcgen05
UWC_DEVI void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
UWC_DEVI void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
UWC_DEVI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
UWC_DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
UWC_DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile written by TMA with 128-byte
// swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart (SBO), sm_100 descriptor version 1,
// layout SWIZZLE_128B. Advancing K inside the 128-byte row is done by adding bytes/16 to the
// start-address field (the swizzle is applied on absolute smem address bits).
UWC_DEVI uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::i8: D s32, A and B signed 8-bit, both K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, one CTA. Issued by one thread.
UWC_DEVI void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05 op issued so far by this thread has completed.
UWC_DEVI void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

UWC_DEVI void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
UWC_DEVI void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 lanes x 256 bits, repeated 8 times along columns (64 columns): thread T of the warp gets
// lane (T/4) -> regs 4j+0,4j+1 and lane (T/4 + 8) -> regs 4j+2,4j+3, columns 8j + 2(T%4) + {0,1}.
// This is the mma.sync m16n8 accumulator fragment layout.
UWC_DEVI void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 32 bits, repeated 32 times: thread T gets lane T, columns 0..31 in regs 0..31.
UWC_DEVI void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 32 bits, repeated 16 times: thread T gets lane T, columns 0..15 in regs 0..15.
UWC_DEVI void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

UWC_DEVI void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Fire-and-forget XOR into global memory (performed at L2).
UWC_DEVI void red_xor(uint32_t* addr, uint32_t v) {
  asm volatile("red.relaxed.gpu.global.xor.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

// XOR of 32 words, 3-input XOR per step (LOP3).
UWC_DEVI uint32_t xor32(const uint32_t* r) {
  uint32_t a = r[0] ^ r[1] ^ r[2], b = r[3] ^ r[4] ^ r[5], c = r[6] ^ r[7] ^ r[8], d = r[9] ^ r[10] ^ r[11];
  uint32_t e = r[12] ^ r[13] ^ r[14], f = r[15] ^ r[16] ^ r[17], g = r[18] ^ r[19] ^ r[20], h = r[21] ^ r[22] ^ r[23];
  uint32_t i = r[24] ^ r[25] ^ r[26], j = r[27] ^ r[28] ^ r[29], k = r[30] ^ r[31];
  return (a ^ b ^ c) ^ (d ^ e ^ f) ^ (g ^ h ^ i) ^ (j ^ k);
}
