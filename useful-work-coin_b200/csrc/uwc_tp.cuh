// Peer exchange of the tensor-parallel decode kernels (new: the reference has no tensor parallelism).
//
// Every rank owns one exchange buffer of the same size and layout; each rank maps every peer's
// buffer (CUDA IPC over NVLink) and the kernels write into peers' buffers with plain stores:
//
//   header   epoch (u64) = calls completed on this buffer, done counter (u32) of the running call
//   flags    [2 parities][8 sources][max_slots] u64: the epoch at which a source's slice landed
//   amax     [2][8][max_m] u64: (epoch << 32) | float bits of a source's row absmax
//   data     [2][8][max_m][max_n] int32: a source's partial products
//
// A call reads E = epoch + 1 and uses parity E & 1; its last CTA sets epoch = E. All ranks run the
// same sequence of calls, so E agrees across ranks, and a rank can be at most one call ahead of a
// peer that still reads the other parity (it cannot finish call E + 1 before that peer has sent).
#pragma once
#include <stdint.h>

#include "../../include/uwc_b200.h"

namespace uwc_tp {

constexpr uint64_t kHeader = 256;
constexpr int kMaxWorld = UWC_TP_MAX_WORLD;

struct Layout {
  uint64_t flags, amax, data, total;
  uint32_t max_m, max_n, max_slots;
};

// max_slots: CTAs of one weight-streaming GEMM (128-row blocks x k-splits <= 8).
__host__ __device__ inline Layout layout(uint32_t max_m, uint32_t max_n) {
  Layout L;
  L.max_m = max_m;
  L.max_n = max_n;
  L.max_slots = ((max_n + 127) / 128) * 8;
  L.flags = kHeader;
  L.amax = L.flags + 2ull * kMaxWorld * L.max_slots * 8;
  L.data = L.amax + 2ull * kMaxWorld * max_m * 8;
  L.data = (L.data + 255) & ~255ull;
  L.total = L.data + 2ull * kMaxWorld * max_m * max_n * 4;
  return L;
}

}  // namespace uwc_tp

namespace uwc_tp {

// System-scope release store / acquire load (the flag protocol between GPUs).
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

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

__device__ __forceinline__ uint64_t* flag_slot(uint8_t* base, const Layout& L, int parity, int src, int slot) {
  return reinterpret_cast<uint64_t*>(base + L.flags) + ((uint64_t)parity * kMaxWorld + src) * L.max_slots + slot;
}
__device__ __forceinline__ uint64_t* amax_slot(uint8_t* base, const Layout& L, int parity, int src, int row) {
  return reinterpret_cast<uint64_t*>(base + L.amax) + ((uint64_t)parity * kMaxWorld + src) * L.max_m + row;
}
__device__ __forceinline__ int32_t* data_of(uint8_t* base, const Layout& L, int parity, int src) {
  return reinterpret_cast<int32_t*>(base + L.data) + ((uint64_t)parity * kMaxWorld + src) * L.max_m * L.max_n;
}

// Spins (bounded by timeout_ns of globaltimer) until pred(ld_acquire(p)) holds; returns the value,
// or raises `status` and returns `fallback` on expiry.
template <typename Pred>
__device__ __forceinline__ uint64_t wait_value(const uint64_t* p, Pred pred, uint64_t timeout_ns, uint32_t* status,
                                               uint64_t fallback, bool* ok) {
  uint64_t v = ld_acquire_sys(p);
  if (pred(v)) return v;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    __nanosleep(64);
    v = ld_acquire_sys(p);
    if (pred(v)) return v;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > timeout_ns) {
      if (status) atomicOr(status, UWC_DEV_TIMEOUT);
      *ok = false;
      return fallback;
    }
  }
}

}  // namespace uwc_tp

// Kernel argument form of UwcTP.
struct TPArgs {
  int rank, world;
  uwc_tp::Layout L;
  uint8_t* base[uwc_tp::kMaxWorld];
};
