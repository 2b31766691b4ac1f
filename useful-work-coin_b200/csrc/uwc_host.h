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

// Adds one to the library's count of kernel launches (uwc_launch_count); called after each launch.
void uwc_count_launch();

// Number of SMs of the current device (cached).
int uwc_num_sms();

// 2D K-major int8 tensor map: `rows` x `cols` bytes, row stride `ld` bytes, box `box_cols` x
// `box_rows`, 128-byte swizzle, out-of-bounds reads as zero. Returns UWC_OK or an error code.
int uwc_make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_rows, uint32_t box_cols);

// Library-internal launchers shared between translation units (not part of the C ABI).
// uwc_noise_uniform that also zeroes a second int32 range (a win counter beside maxabs).
int uwc_noise_uniform_zero2(int8_t* out, uint64_t nbytes, const uint32_t* label, const uint32_t* key,
                            int32_t* zero_me, int zero_n, int32_t* zero2, int zero2_n, void* stream);
// uwc_proj_corr that also copies E (rows x r int8) into corr[li][row][ecopy_off + j] for every limb.
int uwc_proj_corr_ecopy(const int32_t* proj, int rows, int r, int8_t* corr, int corr_off, int32_t* maxabs, int lmax,
                        const int8_t* E, int ecopy_off, void* stream);

// The weight-streaming GEMM (stream_gemm.cu): whether a shape takes it, and its test switches
// (programmatic dependent launch on / off; the bound of its waits, 0 = default).
bool uwc_stream_gemm_fits(int m, int n, int k);
void uwc_stream_set_pdl(int on);
// Programmatic dependent launch of the few-row quantizers (detq.cu) on / off.
void uwc_row_set_pdl(int on);
void uwc_stream_set_wait_ns(uint64_t ns);

// The kernel form of a UwcTP (tp.cu), checked against a call of m rows and n columns.
struct TPArgs;
int uwc_tp_args(const UwcTP* tp, int m, int n, TPArgs* out);

// The bound of device-side waits set by UWC_HOOK_WAIT_NS (0: the default).
uint64_t uwc_wait_ns();

// The smallest world size whose GEMM exchange runs as reduce-scatter + all-gather (tp.cu; default 8).
void uwc_tp_set_two_phase_min(int world);
int uwc_tp_two_phase_min();
