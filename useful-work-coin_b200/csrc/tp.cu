// Exchange buffers of the tensor-parallel decode kernels: allocation and CUDA IPC mapping.
#include <atomic>
#include <cstring>

#include "uwc_device.cuh"
#include "uwc_host.h"
#include "uwc_tp.cuh"

extern "C" uint64_t uwc_tp_buffer_bytes(int max_m, int max_n) {
  if (max_m <= 0 || max_n <= 0) return 0;
  return uwc_tp::layout((uint32_t)max_m, (uint32_t)max_n).total;
}

extern "C" int uwc_tp_alloc(int max_m, int max_n, void** buf) {
  if (!buf || max_m <= 0 || max_n <= 0 || max_m > 65535 || max_n > (1 << 20)) return UWC_ERR_ARG;
  UWC_CHECK_DEVICE();
  const uint64_t bytes = uwc_tp_buffer_bytes(max_m, max_n);
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return UWC_ERR_CUDA;
  }
  *buf = p;
  return UWC_OK;
}

extern "C" int uwc_tp_free(void* buf) {
  if (!buf) return UWC_ERR_ARG;
  return cudaFree(buf) == cudaSuccess ? UWC_OK : (cudaGetLastError(), UWC_ERR_CUDA);
}

extern "C" int uwc_ipc_handle(const void* buf, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == UWC_IPC_HANDLE_BYTES, "IPC handle size");
  if (!buf || !handle) return UWC_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(buf)) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  std::memcpy(handle, &h, sizeof(h));
  return UWC_OK;
}

extern "C" int uwc_ipc_open(const void* handle, void** peer_buf) {
  if (!handle || !peer_buf) return UWC_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  return UWC_OK;
}

extern "C" int uwc_ipc_close(void* peer_buf) {
  if (!peer_buf) return UWC_ERR_ARG;
  return cudaIpcCloseMemHandle(peer_buf) == cudaSuccess ? UWC_OK : (cudaGetLastError(), UWC_ERR_CUDA);
}

namespace {
std::atomic<int> g_two_phase_min{8};
}
void uwc_tp_set_two_phase_min(int world) { g_two_phase_min.store(world); }
int uwc_tp_two_phase_min() { return g_two_phase_min.load(); }

// The kernel form of a UwcTP, checked against the call's shape.
int uwc_tp_args(const UwcTP* tp, int m, int n, TPArgs* out) {
  if (!tp || tp->world < 1 || tp->world > UWC_TP_MAX_WORLD || tp->rank < 0 || tp->rank >= tp->world) return UWC_ERR_ARG;
  if (m > tp->max_m || n > tp->max_n) return UWC_ERR_SHAPE;
  out->rank = tp->rank;
  out->world = tp->world;
  out->two_phase = tp->world >= uwc_tp_two_phase_min() ? 1 : 0;
  out->L = uwc_tp::layout((uint32_t)tp->max_m, (uint32_t)tp->max_n);
  for (int r = 0; r < uwc_tp::kMaxWorld; r++) {
    out->base[r] = r < tp->world ? static_cast<uint8_t*>(tp->base[r]) : nullptr;
    if (r < tp->world && (!tp->base[r] || ((uintptr_t)tp->base[r] & 255))) return UWC_ERR_ARG;
  }
  return UWC_OK;
}

namespace {
// Every rank stores a tagged word into every rank's buffer and polls its own until all ranks'
// words of this call have landed: the ranks leave within about one NVLink write latency.
__global__ void k_tp_barrier(TPArgs tp, uint32_t* status, uint64_t wait_ns) {
  pdl_wait();
  uint8_t* const mine = tp.base[tp.rank];
  const uint64_t E = uwc_tp::call_epoch(mine);
  const int par = (int)(E & 1), p = threadIdx.x;
  if (p < tp.world) {
    uwc_tp::st_sys(uwc_tp::amax_slot(tp.base[p], tp.L, par, tp.rank, 0), uwc_tp::tagged(E, 1u));
    bool ok = true;
    uwc_tp::wait_tagged(uwc_tp::amax_slot(mine, tp.L, par, p, 0), E, uwc_tp::now_ns() + wait_ns, status, &ok);
  }
  __syncthreads();
  if (threadIdx.x == 0) uwc_tp::call_end(mine, E, gridDim.x);
}
}  // namespace

extern "C" int uwc_tp_barrier(const UwcTP* tp, void* stream) {
  TPArgs args;
  const int rc = uwc_tp_args(tp, 1, 0, &args);
  if (rc != UWC_OK) return rc;
  UWC_CHECK_DEVICE();
  const uint64_t ns = uwc_wait_ns();
  k_tp_barrier<<<1, 32, 0, (cudaStream_t)stream>>>(args, uwc_status_ptr(), ns ? ns : uwc_tp::kWaitNs);
  uwc_count_launch();
  return uwc_launch_status();
}
