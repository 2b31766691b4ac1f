// Host-side helpers of the C ABI: device capability check, launch status, TMA descriptors.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/uwc_b200.h"

// Returns UWC_OK when the current device is sm_100 (B200 / GB200), cached per device.
int uwc_check_device();
#define UWC_CHECK_DEVICE()            \
  do {                                \
    int _rc = uwc_check_device();     \
    if (_rc != UWC_OK) return _rc;    \
  } while (0)

// UWC_OK, or UWC_ERR_CUDA if the last launch failed (the error is cleared and remembered).
int uwc_launch_status();

// Device address of the library's status word on the current device (cached), or nullptr.
uint32_t* uwc_status_ptr();

// Number of SMs of the current device (cached).
int uwc_num_sms();

// 2D K-major int8 tensor map: `rows` x `cols` bytes, row stride `ld` bytes, box `box_cols` x
// `box_rows`, 128-byte swizzle, out-of-bounds reads as zero. Returns UWC_OK or an error code.
int uwc_make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_rows, uint32_t box_cols);
