// Host plumbing of the C ABI: device checks, launch status, TMA descriptor encoding, status words.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "uwc_device.cuh"
#include "uwc_host.h"

// Device status word: sticky error bits raised by kernels (bounded waits that ran out).
__device__ uint32_t g_uwc_status = 0;

namespace {
constexpr int kMaxDevices = 64;
int g_dev_ok[kMaxDevices];   // 0 unknown, 1 sm_100, -1 other
int g_dev_sms[kMaxDevices];
uint32_t* g_dev_status[kMaxDevices];
std::mutex g_mu;
std::atomic<uint64_t> g_launches{0};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  if (*dev < 0 || *dev >= kMaxDevices) return UWC_ERR_DEVICE;
  return UWC_OK;
}
}  // namespace

int uwc_check_device() {
  int dev;
  int rc = current_device(&dev);
  if (rc != UWC_OK) return rc;
  int ok = g_dev_ok[dev];
  if (ok == 0) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      cudaGetLastError();
      return UWC_ERR_CUDA;
    }
    ok = (prop.major == 10 && prop.minor == 0) ? 1 : -1;
    g_dev_sms[dev] = prop.multiProcessorCount;
    g_dev_ok[dev] = ok;
  }
  return ok == 1 ? UWC_OK : UWC_ERR_DEVICE;
}

int uwc_num_sms() {
  int dev = 0;
  if (current_device(&dev) != UWC_OK) return 148;
  if (g_dev_sms[dev] == 0) uwc_check_device();
  return g_dev_sms[dev] > 0 ? g_dev_sms[dev] : 148;
}

uint32_t* uwc_status_ptr() {
  int dev = 0;
  if (current_device(&dev) != UWC_OK) return nullptr;
  if (!g_dev_status[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_uwc_status) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    g_dev_status[dev] = static_cast<uint32_t*>(p);
  }
  return g_dev_status[dev];
}

void uwc_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int uwc_launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? UWC_OK : UWC_ERR_CUDA;
}

int uwc_make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_rows, uint32_t box_cols) {
  if (((uintptr_t)base) & 15 || ld % 16) return UWC_ERR_ALIGN;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn) {
        cudaGetLastError();
        return UWC_ERR_CUDA;
      }
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? UWC_OK : UWC_ERR_CUDA;
}

extern "C" {

int uwc_version(void) { return 200; }

uint64_t uwc_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* uwc_status_string(int code) {
  switch (code) {
    case UWC_OK: return "ok";
    case UWC_ERR_ARG: return "bad argument";
    case UWC_ERR_SHAPE: return "shape precondition violated";
    case UWC_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case UWC_ERR_CUDA: return "CUDA error";
    case UWC_ERR_DEVICE: return "device is not sm_100 (B200)";
    case UWC_ERR_SCRATCH: return "scratch buffer too small";
    default: return "unknown status";
  }
}

int uwc_device_status(uint32_t* status_out, int clear) {
  if (!status_out) return UWC_ERR_ARG;
  UWC_CHECK_DEVICE();
  uint32_t v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpyFromSymbol(&v, g_uwc_status, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  *status_out = v;
  if (clear) {
    const uint32_t z = 0;
    if (cudaMemcpyToSymbol(g_uwc_status, &z, sizeof(z)) != cudaSuccess) {
      cudaGetLastError();
      return UWC_ERR_CUDA;
    }
  }
  return UWC_OK;
}

}  // extern "C"
