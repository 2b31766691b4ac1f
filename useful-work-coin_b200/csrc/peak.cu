// The tensor core's int8 rate on this device, measured: back-to-back tcgen05.mma kind::i8 issued
// by one thread per SM from shared-memory tiles that never change, into two TMEM accumulators in
// turn. No TMA, no epilogue, no hand-offs: the denominator a hashed GEMM's tensor work can at most
// reach on this GPU at its current clocks. Used by bench.py for the roofline (no reference
// counterpart: the reference quotes no int8 peak).
#include "uwc_device.cuh"
#include "uwc_host.h"

namespace {

constexpr int kPeakThreads = 128;
constexpr int kPeakA = 128 * 128;   // one 128 x 128-byte A stage (SW128 K-major)
constexpr int kPeakB = 256 * 128;   // one 256 x 128-byte B stage

__global__ void __launch_bounds__(kPeakThreads, 1) k_peak_i8(int iters, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kPeakA + kPeakB) / 16; i += kPeakThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0x01010101u * (i & 7), 0x02020202u, 0, 0x7f7f7f7fu);
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the operand writes, for the tensor core
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  if (warp == 0) {
    if (elect_one()) {
      const uint32_t a = smem_u32(smem), b = a + kPeakA;
      const uint64_t ad = sdesc_sw128(a), bd = sdesc_sw128(b);
      constexpr uint32_t id = idesc_i8(128, 256);
      for (int it = 0; it < iters; it++) {
        // one 128-byte K stage per accumulator, accumulators alternating (as a GEMM's units do)
#pragma unroll
        for (int acc = 0; acc < 2; acc++)
#pragma unroll
          for (int ks = 0; ks < 4; ks++) mma_i8(tmem + acc * 256, ad + 2 * ks, bd + 2 * ks, id, (it | ks) ? 1u : 0u);
      }
      mma_commit(&done);
    }
    __syncwarp();
    mbar_wait(&done, 0, &abort_flag, status);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace

// iters rounds of 8 MMAs (M 128, N 256, K 32 each) per CTA, one CTA per SM on `stream`; the caller
// times the launch with events. int8 operations per launch: uwc_peak_i8_ops(iters).
extern "C" double uwc_peak_i8_ops(int iters) {
  return 2.0 * 128.0 * 256.0 * 32.0 * 8.0 * (double)iters * (double)uwc_num_sms();
}

extern "C" int uwc_peak_i8(int iters, void* stream) {
  if (iters <= 0 || iters > (1 << 17)) return UWC_ERR_ARG;   // <= ~0.1 s, far inside the 1 s wait bound
  UWC_CHECK_DEVICE();
  const int smem = kPeakA + kPeakB + 1024;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(k_peak_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      cudaGetLastError();
      return UWC_ERR_CUDA;
    }
    configured[dev] = 1;
  }
  k_peak_i8<<<uwc_num_sms(), kPeakThreads, smem, (cudaStream_t)stream>>>(iters, uwc_status_ptr());
  uwc_count_launch();
  return uwc_launch_status();
}
