// Weight-streaming int8 GEMM for decode-sized m (sm_100a): out (m x n) = X (m x k) W (n x k)^T.
//
// When m is small the product is bound by reading W once from HBM. The operands swap roles on the
// tensor core: a 128-row tile of W is the MMA's M side and all m rows of X (padded to MP = 16, 32
// or 64) its N side, so D^T = W X^T accumulates in MP columns of tensor memory. Each CTA owns one
// (128-row block of W, k-range) unit; the k-splits of a row block form one thread-block cluster
// and add their partial tiles through distributed shared memory (integer sums: exact in any order),
// each CTA finishing a slice of the block's rows. There is no global accumulator, no memset and no
// second pass, and the epilogue applies the deterministic linear's output step in place:
//
//   UWC_SEPI_I32     int32 q W^T                                  runtime/detrt/qwen3.py:106-119
//   UWC_SEPI_F32     fmul(fmul(float(acc), s_x), s_w)             runtime/detrt/qwen3.py:125
//   UWC_SEPI_BF16    the same, rounded to bf16 (RNE)               miner/ampere/uwc_ampere/model.py:117
//   UWC_SEPI_RESID   fadd(x, deq(acc)) (row-parallel + residual)  runtime/detgpu/kernels.py:346-354
//   UWC_SEPI_SWIGLU  fmul(det_silu(deq(gate)), deq(up)) of a     runtime/detgpu/kernels.py:356-396
//                    gate/up weight (I gate rows, then I up rows):
//                    each tile stacks 64 gate rows over their 64
//                    up rows (two 64-row copies per stage)
//
// Warp roles (192 threads): warp 0 issues the TMA copies, warp 1 the MMAs, warps 2..5 read the
// accumulator (warp w reads tensor-memory lanes 32 (w % 4) ..) and run the reduction and epilogue.
// Every mbarrier wait is bounded; an expired wait raises UWC_DEV_TIMEOUT and the CTA unwinds.
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>

#include "det_math.cuh"
#include "uwc_device.cuh"
#include "uwc_host.h"
#include "uwc_tp.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int kSThreads = 192;
constexpr int kSKB = 128;            // k bytes per stage (one 128-byte swizzle row)
constexpr int kSRows = 128;          // W rows per tile
constexpr int kSMaxSplit = 8;        // portable cluster size

struct SParams {
  int m, n, k;
  int kblocks, ksplit;               // k-blocks of 128 bytes; CTAs (cluster size) per row block
  int epi;
  const float* x_scale;              // per row of X (m)
  const float* w_scale;              // per row of W (n)
  const float* resid;                // UWC_SEPI_RESID: x (m x n fp32) or nullptr
  void* out;
  int ldo;                           // output row stride in elements (n, or n / 2 for SWIGLU)
  int half;                          // SWIGLU: I = n / 2, the first up row; 0 otherwise
  int early_w;                       // W may be read before the previous kernel has finished
  int tp_on;                         // sum the int32 product over the ranks of `tp` first
  TPArgs tp;
  uint32_t* status;
  uint64_t wait_ns;
};

template <int MP>
struct SCfg {
  static constexpr int W_BYTES = kSRows * kSKB;                 // 16 KiB
  static constexpr int X_BYTES = MP * kSKB;
  static constexpr int STAGE = W_BYTES + X_BYTES;
  // about 100 KiB of stages: two CTAs fit on one SM
  static constexpr int NST = MP == 16 ? 6 : (MP == 32 ? 5 : 4);
  static constexpr int PART_BYTES = kSRows * MP * 4;            // the partial tile, [t][row]
  static_assert(PART_BYTES <= NST * STAGE, "partial tile reuses the stage ring");
  static constexpr int BAR_OFF = NST * STAGE;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;              // + barriers, + 1 KiB alignment slack
  static constexpr uint32_t TCOLS = MP < 32 ? 32 : MP;           // tensor-memory columns (power of 2, >= 32)
};

struct SBars {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint32_t bf16_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

__device__ __forceinline__ bool sw_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        const SParams& p) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status, p.wait_ns));
}

}  // namespace

namespace {

// Programmatic dependent launch: this kernel may start while the previous kernel in the stream
// still runs. Everything before pdl_wait() touches only W and this CTA's own state; X, the scales,
// the residual and the output are read or written after it.

template <int MP>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, uint32_t* v) {
  if constexpr (MP == 16) {
    tmem_ld_32x32b_x16(taddr, v);
  } else if constexpr (MP == 32) {
    tmem_ld_32x32b_x32(taddr, v);
  } else {
    tmem_ld_32x32b_x32(taddr, v);
    tmem_ld_32x32b_x32(taddr + 32, v + 32);
  }
}

// One output element of the epilogue: the summed accumulator of W row j (block-relative jj in the
// row block rb) and X row t.
__device__ __forceinline__ void store_one(const SParams& p, int t, int j, int32_t acc) {
  const uint64_t o = (uint64_t)t * p.ldo + j;
  switch (p.epi) {
    case UWC_SEPI_I32:
      static_cast<int32_t*>(p.out)[o] = acc;
      return;
    case UWC_SEPI_F32:
      static_cast<float*>(p.out)[o] = deq(acc, p.x_scale[t], __ldg(p.w_scale + j));
      return;
    case UWC_SEPI_BF16:
      static_cast<uint16_t*>(p.out)[o] = (uint16_t)bf16_bits(deq(acc, p.x_scale[t], __ldg(p.w_scale + j)));
      return;
    default: {  // UWC_SEPI_RESID
      const float y = deq(acc, p.x_scale[t], __ldg(p.w_scale + j));
      static_cast<float*>(p.out)[o] = p.resid ? __fadd_rn(p.resid[(uint64_t)t * p.n + j], y) : y;
      return;
    }
  }
}

// The stage's 128 W rows: rows 128 rb .. (one 128-row box), or for SWIGLU gate rows 64 rb .. above
// up rows half + 64 rb .. (two 64-row boxes; the upper one lands 8 KiB in, on a swizzle atom).
__device__ __forceinline__ void load_w(uint8_t* sW, const CUtensorMap* tmW, uint64_t* bar, int x, int rb, int half) {
  if (half) {
    tma_load_2d(sW, tmW, bar, x, rb * (kSRows / 2));
    tma_load_2d(sW + (kSRows / 2) * kSKB, tmW, bar, x, half + rb * (kSRows / 2));
  } else {
    tma_load_2d(sW, tmW, bar, x, rb * kSRows);
  }
}

template <int MP>
__global__ void __launch_bounds__(kSThreads, 2)
    k_stream_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const SParams p) {
  using C = SCfg<MP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SBars* bars = reinterpret_cast<SBars*>(smem + C::BAR_OFF);
  volatile int* abort_flag = &bars->abort_flag;
  int32_t* part = reinterpret_cast<int32_t*>(smem);          // [t][row], after the main loop
  cg::cluster_group cluster = cg::this_cluster();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = (int)cluster.block_rank(), rb = blockIdx.y;
  const int kb0 = (int)((long long)ks * p.kblocks / p.ksplit);
  const int nkb = (int)((long long)(ks + 1) * p.kblocks / p.ksplit) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NST; s++) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    bars->abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::TCOLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    const bool leader = elect_one();
    // the first ring's worth of W, before the previous kernel has finished when the caller says W
    // is not written by it (UWC_SEPI_EARLY_W), then X behind the grid dependency
    const int pre = min(nkb, C::NST);
    if (!p.early_w) pdl_wait();
    if (leader) {
      for (int b = 0; b < pre; b++) {
        mbar_expect_tx(&bars->full[b], C::STAGE);
        load_w(smem + b * C::STAGE, &tmW, &bars->full[b], (kb0 + b) * kSKB, rb, p.half);
      }
    }
    pdl_wait();
    if (leader)
      for (int b = 0; b < pre; b++)
        tma_load_2d(smem + b * C::STAGE + C::W_BYTES, &tmX, &bars->full[b], (kb0 + b) * kSKB, 0);
    for (int b = pre; b < nkb && ok; b++) {
      const int s = b % C::NST;
      const uint32_t ph = (b / C::NST) & 1;
      ok = sw_wait(&bars->empty[s], ph ^ 1, abort_flag, p);
      if (!ok) break;
      if (leader) {
        uint8_t* sW = smem + s * C::STAGE;
        mbar_expect_tx(&bars->full[s], C::STAGE);
        load_w(sW, &tmW, &bars->full[s], (kb0 + b) * kSKB, rb, p.half);
        tma_load_2d(sW + C::W_BYTES, &tmX, &bars->full[s], (kb0 + b) * kSKB, 0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    pdl_wait();
    const bool leader = elect_one();
    constexpr uint32_t idesc = idesc_i8(kSRows, MP);
    for (int b = 0; b < nkb && ok; b++) {
      const int s = b % C::NST;
      ok = sw_wait(&bars->full[s], (b / C::NST) & 1, abort_flag, p);
      if (!ok) break;
      tc_fence_after();
      if (leader) {
        const uint32_t aW = smem_u32(smem + s * C::STAGE);
        const uint64_t ad = sdesc_sw128(aW), bd = sdesc_sw128(aW + C::W_BYTES);
#pragma unroll
        for (int kk = 0; kk < kSKB / 32; kk++) mma_i8(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (b | kk) ? 1u : 0u);
        mma_commit(&bars->empty[s]);
      }
      __syncwarp();
    }
    if (leader) mma_commit(&bars->acc_full);
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- accumulator read-out
    pdl_wait();
    const int q = warp & 3, row = 32 * q + lane;
    ok = sw_wait(&bars->acc_full, 0, abort_flag, p);
    if (ok) {
      tc_fence_after();
      uint32_t v[MP];
      tmem_ld_row<MP>(tmem + ((uint32_t)(32 * q) << 16), v);
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < MP; t++) part[t * kSRows + row] = (int32_t)v[t];
    }
    tc_fence_before();
  }
  // every CTA of the cluster has its partial tile in shared memory (or has given up)
  pdl_trigger();
  cluster.sync();
  if (warp == 1) tmem_dealloc(tmem, C::TCOLS);

  // ---------------------------------------------------------------- cluster reduction + epilogue
  // CTA `ks` finishes rows [r0, r1) of the block (SWIGLU: gate rows r0..r1-1 of the first 64 and
  // their up rows + 64), summing the cluster's partial tiles in rank order.
  {
    const bool live = !*abort_flag;
    const int32_t* peer[kSMaxSplit];
#pragma unroll
    for (int c = 0; c < kSMaxSplit; c++) peer[c] = c < p.ksplit ? cluster.map_shared_rank(part, c) : part;
    const bool swiglu = p.epi == UWC_SEPI_SWIGLU;
    const int span = swiglu ? kSRows / 2 : kSRows;
    const int r0 = ks * span / p.ksplit, nr = (ks + 1) * span / p.ksplit - r0;
    const int total = nr * p.m;
    auto cluster_sum = [&](int t, int jj, int32_t& acc_up) {
      int32_t acc = 0;
      acc_up = 0;
#pragma unroll
      for (int c = 0; c < kSMaxSplit; c++) {
        if (c < p.ksplit) {
          acc += peer[c][t * kSRows + jj];
          if (swiglu) acc_up += peer[c][t * kSRows + jj + kSRows / 2];
        }
      }
      return acc;
    };
    if (p.tp_on) {
      // The ranks' partial products of this slice, as 8-byte words tagged with the call's epoch.
      // One-shot: every rank sends its partials to every rank, each sums them in rank order.
      // Two-phase (many ranks): the slot's owner rank receives the partials, sums them in rank
      // order and sends the total to every rank: 2 (N - 1) / N of the product per rank instead of
      // N - 1.
      uint8_t* const mine = p.tp.base[p.tp.rank];
      const uint64_t E = uwc_tp::call_epoch(mine);
      const int par = (int)(E & 1), world = p.tp.world;
      const int owner = (rb * p.ksplit + ks) % world;
      const bool two = p.tp.two_phase != 0;
      const uint32_t ldn = p.tp.L.max_n;
      for (int idx = threadIdx.x; idx < total; idx += kSThreads) {
        const int t = idx / nr, jj = r0 + (idx - t * nr), j = rb * kSRows + jj;
        int32_t up;
        const int32_t acc = live ? cluster_sum(t, jj, up) : 0;
        if (j >= p.n) continue;
        const uint64_t w = uwc_tp::tagged(E, (uint32_t)acc), off = (uint64_t)t * ldn + j;
        if (two) {
          uwc_tp::st_sys(uwc_tp::data_of(p.tp.base[owner], p.tp.L, par, p.tp.rank) + off, w);
        } else {
          for (int d = 0; d < world; d++) uwc_tp::st_sys(uwc_tp::data_of(p.tp.base[d], p.tp.L, par, p.tp.rank) + off, w);
        }
      }
      // receive: kPoll items per thread at a time, each source's words loaded together (independent
      // loads in flight), then only stale words polled again
      constexpr int kPoll = 4;
      bool ok = true;
      const uint64_t deadline = uwc_tp::now_ns() + p.wait_ns;
      auto sum_sources = [&](const uint64_t* off, const bool* use, int32_t* acc) {
        for (int src = 0; src < world; src++) {
          const uint64_t* d = uwc_tp::data_of(mine, p.tp.L, par, src);
          uint64_t w[kPoll];
#pragma unroll
          for (int c = 0; c < kPoll; c++) w[c] = use[c] ? uwc_tp::ld_sys(d + off[c]) : 0;
#pragma unroll
          for (int c = 0; c < kPoll; c++) {
            if (!use[c]) continue;
            const uint32_t v = (uint32_t)(w[c] >> 32) == (uint32_t)E
                                   ? (uint32_t)w[c]
                                   : uwc_tp::wait_tagged(d + off[c], E, deadline, p.status, &ok);
            acc[c] += (int32_t)v;
          }
        }
      };
      for (int i0 = threadIdx.x; i0 < total; i0 += kSThreads * kPoll) {
        uint64_t off[kPoll];
        bool use[kPoll];
        int32_t acc[kPoll];
#pragma unroll
        for (int c = 0; c < kPoll; c++) {
          const int idx = i0 + c * kSThreads;
          const int t = idx / nr, j = rb * kSRows + r0 + (idx - t * nr);
          use[c] = idx < total && j < p.n;
          off[c] = use[c] ? (uint64_t)t * ldn + j : 0;
          acc[c] = 0;
        }
        if (!two) {
          sum_sources(off, use, acc);
        } else {
          if (owner == p.tp.rank) {
            sum_sources(off, use, acc);
#pragma unroll
            for (int c = 0; c < kPoll; c++)
              if (use[c])
                for (int d = 0; d < world; d++)
                  if (d != p.tp.rank)
                    uwc_tp::st_sys(uwc_tp::sum_of(p.tp.base[d], p.tp.L, par) + off[c], uwc_tp::tagged(E, (uint32_t)acc[c]));
          } else {
            const uint64_t* d = uwc_tp::sum_of(mine, p.tp.L, par);
            uint64_t w[kPoll];
#pragma unroll
            for (int c = 0; c < kPoll; c++) w[c] = use[c] ? uwc_tp::ld_sys(d + off[c]) : 0;
#pragma unroll
            for (int c = 0; c < kPoll; c++)
              if (use[c])
                acc[c] = (int32_t)((uint32_t)(w[c] >> 32) == (uint32_t)E
                                       ? (uint32_t)w[c]
                                       : uwc_tp::wait_tagged(d + off[c], E, deadline, p.status, &ok));
          }
        }
#pragma unroll
        for (int c = 0; c < kPoll; c++) {
          if (!use[c]) continue;
          const int idx = i0 + c * kSThreads;
          const int t = idx / nr;
          store_one(p, t, rb * kSRows + r0 + (idx - t * nr), acc[c]);
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) uwc_tp::call_end(mine, E, gridDim.x * gridDim.y);
    } else if (live) {
      for (int idx = threadIdx.x; idx < total; idx += kSThreads) {
        const int t = idx / nr, jj = r0 + (idx - t * nr);
        int32_t acc_up;
        const int32_t acc = cluster_sum(t, jj, acc_up);
        if (swiglu) {
          const int f = rb * (kSRows / 2) + jj;
          if (f < p.half) {
            const float xs = p.x_scale[t];
            const float g = deq(acc, xs, __ldg(p.w_scale + f));
            const float u = deq(acc_up, xs, __ldg(p.w_scale + p.half + f));
            static_cast<float*>(p.out)[(uint64_t)t * p.ldo + f] = det_swiglu(g, u);
          }
        } else {
          const int j = rb * kSRows + jj;
          if (j < p.n) store_one(p, t, j, acc);
        }
      }
    }
  }
  // peers keep their shared memory until every CTA of the cluster has read it
  cluster.sync();
}

template <int MP>
int launch_stream(const SParams& p, const CUtensorMap& tw, const CUtensorMap& tx, int nrb, cudaStream_t st,
                  bool pdl) {
  using C = SCfg<MP>;
  static std::atomic<int> configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return UWC_ERR_CUDA;
  if (!configured[dev].load()) {
    if (cudaFuncSetAttribute(k_stream_gemm<MP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess) {
      cudaGetLastError();
      return UWC_ERR_CUDA;
    }
    configured[dev].store(1);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ksplit, nrb, 1);
  cfg.blockDim = dim3(kSThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.ksplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_stream_gemm<MP>, tw, tx, p);
  uwc_count_launch();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  return uwc_launch_status();
}

std::atomic<int> g_stream_pdl{1};
std::atomic<uint64_t> g_stream_wait_ns{0};

// k-splits per 128-row block: enough CTAs to cover the SMs once, at least four k-blocks each, at most
// a portable cluster. (Measured along the C5 decode chain: covering the SMs twice with clusters of 8
// is faster for one GEMM alone but slower in the chain, where the quantizers' CTAs hold SM space.)
int pick_split(int nrb, int kblocks) {
  const int want = (uwc_num_sms() + nrb - 1) / nrb;
  return std::max(1, std::min({want, kSMaxSplit, std::max(1, kblocks / 4)}));
}

}  // namespace

void uwc_stream_set_pdl(int on) { g_stream_pdl.store(on ? 1 : 0); }
void uwc_stream_set_wait_ns(uint64_t ns) { g_stream_wait_ns.store(ns); }

bool uwc_stream_gemm_fits(int m, int n, int k) { return m >= 1 && m <= 64 && n >= 1 && k >= 16 && k % 16 == 0; }

namespace {
int stream_call(const int8_t* X, const int8_t* W, int m, int n, int k, const float* x_scale, const float* w_scale,
                const float* resid, void* out, int epi, const UwcTP* tp, void* stream) {
  const int early_w = (epi & UWC_SEPI_EARLY_W) ? 1 : 0;
  epi &= ~UWC_SEPI_EARLY_W;
  if (!X || !W || !out || epi < UWC_SEPI_I32 || epi > UWC_SEPI_SWIGLU) return UWC_ERR_ARG;
  if (epi != UWC_SEPI_I32 && (!x_scale || !w_scale)) return UWC_ERR_ARG;
  if (resid && epi != UWC_SEPI_RESID) return UWC_ERR_ARG;
  if (tp && epi == UWC_SEPI_SWIGLU) return UWC_ERR_ARG;
  if (!uwc_stream_gemm_fits(m, n, k)) return UWC_ERR_SHAPE;
  if (epi == UWC_SEPI_SWIGLU && n % kSRows) return UWC_ERR_SHAPE;   // I % 64 == 0
  if ((((uintptr_t)X) | ((uintptr_t)W)) & 15) return UWC_ERR_ALIGN;
  SParams p{};
  if (tp) {
    const int rc = uwc_tp_args(tp, m, n, &p.tp);
    if (rc != UWC_OK) return rc;
    p.tp_on = 1;
  }
  UWC_CHECK_DEVICE();
  p.m = m; p.n = n; p.k = k; p.epi = epi;
  p.x_scale = x_scale; p.w_scale = w_scale; p.resid = resid; p.out = out;
  p.ldo = epi == UWC_SEPI_SWIGLU ? n / 2 : n;
  p.half = epi == UWC_SEPI_SWIGLU ? n / 2 : 0;
  p.early_w = early_w;
  p.status = uwc_status_ptr();
  const uint64_t ns = g_stream_wait_ns.load();
  p.wait_ns = ns ? ns : (tp ? uwc_tp::kWaitNs : UWC_WAIT_TIMEOUT_NS);
  p.kblocks = (k + kSKB - 1) / kSKB;
  const int nrb = (n + kSRows - 1) / kSRows;
  p.ksplit = pick_split(nrb, p.kblocks);
  // the exchange waits for the peers' CTAs of the same call: every CTA must be resident (two per SM)
  if (tp && (long long)nrb * p.ksplit > 2LL * uwc_num_sms()) return UWC_ERR_SHAPE;
  const int MP = m <= 16 ? 16 : (m <= 32 ? 32 : 64);
  CUtensorMap tw, tx;
  int rc = uwc_make_tmap_2d(&tw, W, (uint64_t)n, (uint64_t)k, (uint64_t)k, p.half ? kSRows / 2 : kSRows, kSKB);
  if (rc == UWC_OK) rc = uwc_make_tmap_2d(&tx, X, (uint64_t)m, (uint64_t)k, (uint64_t)k, MP, kSKB);
  if (rc != UWC_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = g_stream_pdl.load() != 0;
  if (MP == 16) return launch_stream<16>(p, tw, tx, nrb, st, pdl);
  if (MP == 32) return launch_stream<32>(p, tw, tx, nrb, st, pdl);
  return launch_stream<64>(p, tw, tx, nrb, st, pdl);
}
}  // namespace

extern "C" int uwc_gemm_stream(const int8_t* X, const int8_t* W, int m, int n, int k, const float* x_scale,
                               const float* w_scale, const float* resid, void* out, int epi, void* stream) {
  return stream_call(X, W, m, n, k, x_scale, w_scale, resid, out, epi, nullptr, stream);
}

extern "C" int uwc_gemm_stream_tp(const int8_t* X, const int8_t* W, int m, int n, int k, const float* x_scale,
                                  const float* w_scale, const float* resid, void* out, int epi, const UwcTP* tp,
                                  void* stream) {
  if (!tp) return UWC_ERR_ARG;
  return stream_call(X, W, m, n, k, x_scale, w_scale, resid, out, epi, tp, stream);
}
