// Host launcher for the reference's own GPU NoisyGEMM, so it can be timed on the same B200 and the
// same inputs as this library's kernel. The kernel source is NOT part of this repository: the build
// recipe (baseline/build_ref_kernel.py) compiles the reference checkout's
// miner/ampere/uwc_ampere/kernels.cu where it lies, by including it through UWC_REF_KERNELS, with
// the reference's default tile configuration (ops.py: CONFIGS["128x3"] = BN 128, 3 stages, MINB 2).
// The launch reproduces ops.gemm (miner/ampere/uwc_ampere/ops.py:185-198): grid (n / BN) * (m / BM),
// BN threads, STAGES * (BM + BN) * BK bytes of dynamic shared memory, the same argument list.
#include <cuda_runtime.h>

#include UWC_REF_KERNELS

extern "C" int ref_noisy_gemm_config(int* bm, int* bn, int* bk) {
  *bm = BM;
  *bn = BN;
  *bk = BK;
  return 0;
}

// Returns the CUDA error of the launch (0 = success); shapes must satisfy the reference's asserts
// (m % BM, n % BN, k % BK, r % BK, k % r all zero), which the caller checks.
extern "C" int ref_noisy_gemm(const void* A, const void* B, int m, int n, int k, int r, const void* corrA,
                              const void* corrB, const void* maxabs, const void* key, const void* target, void* wins,
                              int max_wins, const float* a_scale, const float* b_scale, void* out, int out_mode,
                              int flags, int lmax, void* stream) {
  const int smem = STAGES * (BM + BN) * BK;
  static int configured = 0;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(noisy_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    configured = 1;
  }
  noisy_gemm<<<(n / BN) * (m / BM), NTHREADS, smem, (cudaStream_t)stream>>>(
      (const i8*)A, (const i8*)B, m, n, k, r, (const i8*)corrA, (const i8*)corrB, (const i32*)maxabs, (const u32*)key,
      (const u32*)target, (u32*)wins, max_wins, a_scale, b_scale, out, out_mode, flags, lmax);
  return (int)cudaGetLastError();
}
