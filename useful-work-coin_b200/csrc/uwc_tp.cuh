// Peer exchange of the tensor-parallel decode kernels (new: the reference has no tensor parallelism).
//
// Every rank owns one exchange buffer of the same size and layout; each rank maps every peer's
// buffer (CUDA IPC over NVLink) and the kernels write into peers' buffers with plain stores:
//
//   header   epoch (u64) = calls completed on this buffer, done counter (u32) of the running call
//   amax     [2 parities][8 sources][max_m] u64: (epoch << 32) | float bits of a source's row absmax
//   data     [2][8][max_m][max_n] u64: (epoch << 32) | a source's int32 partial product
//   sum      [2][max_m][max_n] u64: (epoch << 32) | the summed product, from its owner rank
//             (the reduce-scatter + all-gather form of the GEMM's exchange)
//
// Every value carries the epoch of the call that wrote it in the same 8-byte store, so a reader
// polls the value itself: no flags, no fences, one NVLink write latency per exchange.
//
// A call reads E = epoch + 1 and uses parity E & 1; its last CTA sets epoch = E. All ranks run the
// same sequence of calls, so E agrees across ranks, and a rank can be at most one call ahead of a
// peer that still reads the other parity (it cannot finish call E + 1 before that peer has sent).
#pragma once
#include <stdint.h>

#include "../../include/uwc_b200.h"

namespace uwc_tp {

constexpr uint64_t kHeader = 256;
// Default bound of a cross-GPU wait: ranks may reach a call seconds apart (process start, lazy
// module loading, rank-local setup between collectives), so it is longer than the in-GPU waits'.
constexpr uint64_t kWaitNs = 10ull * 1000000000ull;
constexpr int kMaxWorld = UWC_TP_MAX_WORLD;

struct Layout {
  uint64_t amax, data, sum, total;
  uint32_t max_m, max_n;
};

__host__ __device__ inline Layout layout(uint32_t max_m, uint32_t max_n) {
  Layout L;
  L.max_m = max_m;
  L.max_n = max_n;
  L.amax = kHeader;
  L.data = L.amax + 2ull * kMaxWorld * max_m * 8;
  L.data = (L.data + 255) & ~255ull;
  L.sum = L.data + 2ull * kMaxWorld * max_m * max_n * 8;
  L.total = L.sum + 2ull * max_m * max_n * 8;
  return L;
}

}  // namespace uwc_tp

namespace uwc_tp {

// System-scope relaxed 8-byte store / load: single-copy atomic, seen by (and seeing) other GPUs.
__device__ __forceinline__ void st_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The tagged word of epoch E carrying v.
__device__ __forceinline__ uint64_t tagged(uint64_t E, uint32_t v) { return (E << 32) | v; }

__device__ __forceinline__ uint64_t* header_epoch(uint8_t* base) { return reinterpret_cast<uint64_t*>(base); }
__device__ __forceinline__ unsigned* header_done(uint8_t* base) { return reinterpret_cast<unsigned*>(base + 8); }

// The call's epoch E (this buffer's completed calls + 1).
__device__ __forceinline__ uint64_t call_epoch(uint8_t* base) {
  return *reinterpret_cast<volatile uint64_t*>(header_epoch(base)) + 1;
}

// Called by one thread of every CTA at the very end: the last CTA of the grid publishes epoch E.
__device__ __forceinline__ void call_end(uint8_t* base, uint64_t E, unsigned nblocks) {
  __threadfence();
  if (atomicAdd(header_done(base), 1u) == nblocks - 1) {
    *header_done(base) = 0;
    __threadfence();
    *reinterpret_cast<volatile uint64_t*>(header_epoch(base)) = E;
  }
}

__device__ __forceinline__ uint64_t* amax_slot(uint8_t* base, const Layout& L, int parity, int src, int row) {
  return reinterpret_cast<uint64_t*>(base + L.amax) + ((uint64_t)parity * kMaxWorld + src) * L.max_m + row;
}
__device__ __forceinline__ uint64_t* data_of(uint8_t* base, const Layout& L, int parity, int src) {
  return reinterpret_cast<uint64_t*>(base + L.data) + ((uint64_t)parity * kMaxWorld + src) * L.max_m * L.max_n;
}

__device__ __forceinline__ uint64_t* sum_of(uint8_t* base, const Layout& L, int parity) {
  return reinterpret_cast<uint64_t*>(base + L.sum) + (uint64_t)parity * L.max_m * L.max_n;
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The low 32 bits of the tagged word at p once its tag is epoch E. Spins until then or until the
// globaltimer passes `deadline` (then raises UWC_DEV_TIMEOUT in `status`, clears *ok and returns 0;
// later waits of the same thread give up at once).
__device__ __forceinline__ uint32_t wait_tagged(const uint64_t* p, uint64_t E, uint64_t deadline, uint32_t* status,
                                                bool* ok) {
  const uint32_t want = (uint32_t)E;
  uint64_t v = ld_sys(p);
  while ((uint32_t)(v >> 32) != want) {
    if (!*ok) return 0;
    if (now_ns() > deadline) {
      if (status) atomicOr(status, UWC_DEV_TIMEOUT);
      *ok = false;
      return 0;
    }
    v = ld_sys(p);
  }
  return (uint32_t)v;
}

}  // namespace uwc_tp

// Kernel argument form of UwcTP.
struct TPArgs {
  int rank, world;
  int two_phase;   // the GEMM's exchange as reduce-scatter + all-gather (else one-shot)
  uwc_tp::Layout L;
  uint8_t* base[uwc_tp::kMaxWorld];
};
