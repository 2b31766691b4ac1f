/*
 * uwc_b200.h -- C ABI of the B200 (sm_100a) NoisyGEMM library (libuwcb200.so).
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream (as void*, 0 = the legacy
 * default stream), launches asynchronously on that stream and returns an int status (UWC_OK or
 * an UWC_ERR_* code below). No entry point allocates device memory: workspaces are caller-owned
 * and their sizes are queryable. Launch errors are reported by the return code; errors detected
 * inside kernels (a bounded wait that ran out) are sticky bits read with uwc_device_status().
 *
 * Each declaration names the reference interface it replaces (paths inside
 * srivassid/useful-work-coin). The reference launches CUDA C++ kernels through CuPy from
 * miner/ampere/uwc_ampere/ops.py; the Python mirror of that module in this repository
 * (useful-work-coin_b200/uwc_b200/ops.py) binds these functions with ctypes.
 *
 * Threading: like the reference (ops.py:62-70), callers serialize work on one stream per device;
 * the library keeps per-device launch configuration and tensor-map caches guarded by a mutex.
 */
#ifndef UWC_B200_H
#define UWC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host return values) */
#define UWC_OK 0
#define UWC_ERR_ARG 1     /* null pointer where one is required, bad enum value */
#define UWC_ERR_SHAPE 2   /* shape precondition violated (the reference's asserts, ops.py:191-192) */
#define UWC_ERR_ALIGN 3   /* pointer or row stride not 16-byte aligned */
#define UWC_ERR_CUDA 4    /* CUDA runtime / driver error while configuring or launching */
#define UWC_ERR_DEVICE 5  /* current device is not sm_100 (B200) */
#define UWC_ERR_SCRATCH 6 /* caller-provided scratch too small */

/* ---- device status bits (uwc_device_status) */
#define UWC_DEV_TIMEOUT 1u /* a kernel's bounded wait ran out and the kernel unwound */

/* ---- constants shared with the reference (ops.py:26-29, kernels.cu:475-480) */
#define UWC_FLAG_HASH 1
#define UWC_FLAG_DENOISE 2
#define UWC_OUT_NONE 0
#define UWC_OUT_I32 1
#define UWC_OUT_BF16 2
#define UWC_OUT_F32 3 /* new: detrt dequant y = fmul(fmul(float(acc), a_scale[i]), b_scale[j]) (qwen3.py:125) */
#define UWC_WIN_WORDS 10

/* Test hooks of the error path (no counterpart in the reference). UWC_HOOK_WAIT_NS sets the bound of
 * every wait inside the GEMM kernels (value in ns; 0 restores the default of 1 s);
 * UWC_HOOK_WITHHOLD = 1 makes later GEMM launches issue no copies, so their first wait runs out and
 * the kernel unwinds with UWC_DEV_TIMEOUT in uwc_device_status (0 restores normal launches);
 * UWC_HOOK_STREAM_PDL = 0 launches the weight-streaming GEMM and the few-row quantizers without
 * programmatic dependent launch (1, the default, lets them start while the previous kernel of the
 * stream finishes); UWC_HOOK_TP_TWO_PHASE = w (1..9) runs uwc_gemm_stream_tp's exchange as
 * reduce-scatter + all-gather from w ranks on (default 8; 9: never).
 * Process-wide; for tests only. Returns UWC_OK or UWC_ERR_ARG. */
#define UWC_HOOK_WAIT_NS 1
#define UWC_HOOK_WITHHOLD 2
#define UWC_HOOK_STREAM_PDL 3
#define UWC_HOOK_TP_TWO_PHASE 4
int uwc_test_hook(int hook, long long value);

/* Library version (major*10000 + minor*100 + patch). */
int uwc_version(void);

/* Kernels this library has launched in this process (all devices, all threads): a counter the
 * caller reads before and after a region to count the library's launches in it. */
uint64_t uwc_launch_count(void);

/* Human-readable name of a status code. */
const char* uwc_status_string(int code);

/* Sticky device status bits of the current device (UWC_DEV_*). Synchronizes the device.
 * clear != 0 resets them to 0 afterwards. */
int uwc_device_status(uint32_t* status_out, int clear);

/* ---- BLAKE3 commitment ------------------------------------------------------------------
 * Replaces ops.b3_root_and_seed (miner/ampere/uwc_ampere/ops.py:99-118) and the kernels
 * b3_tree_stage1/_mid/_stage2 (kernels.cu:138-244).
 * Keyed BLAKE3 Merkle root of `nbytes` bytes (nbytes % 1024 == 0, > 0) under the 8-word key.
 * If seed_out != NULL also derives Pearl's cert-v3 salted seed
 *   seed = BLAKE3(prefix || BLAKE3_keyed(salt, root || dim_le32 || 0^28))
 * (prefix, salt: 8 words each, device). root_out may be NULL.
 * scratch: device u32 workspace of uwc_b3_scratch_words(nbytes) words. */
uint64_t uwc_b3_scratch_words(uint64_t nbytes);
int uwc_b3_root_and_seed(const void* data, uint64_t nbytes, const uint32_t* key, const uint32_t* prefix,
                         const uint32_t* salt, uint32_t dim, uint32_t* root_out, uint32_t* seed_out,
                         uint32_t* scratch, uint64_t scratch_words, void* stream);

/* Same commitment and seed as uwc_b3_root_and_seed, for callers that cannot allocate device
 * memory (inside CUDA graph capture, foreign-function callers without a device allocator,
 * processes whose device memory is reserved by another framework): no counterpart in the
 * reference. The scratch is a fixed 32 KiB array in the library's device memory, so inputs are
 * limited to uwc_b3_noalloc_max_bytes() (128 MiB); larger ones return UWC_ERR_SCRATCH. No
 * allocation of any kind. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and should come before any stream capture. All calls on a device share
 * the array: calls that overlap on the GPU race and must be serialized by the caller. The looked-up
 * address is cached per device (host threads may make their first calls concurrently) for the life
 * of the device's CUDA context; a caller that resets a device (cudaDeviceReset) calls
 * uwc_b3_noalloc_forget() afterwards. */
uint64_t uwc_b3_noalloc_max_bytes(void);
void uwc_b3_noalloc_forget(void);
int uwc_b3_root_and_seed_noalloc(const void* data, uint64_t nbytes, const uint32_t* key, const uint32_t* prefix,
                                 const uint32_t* salt, uint32_t dim, uint32_t* root_out, uint32_t* seed_out,
                                 void* stream);

/* ---- noise generation ------------------------------------------------------------------
 * Replaces ops.noise_uniform (ops.py:122-125, kernels.cu:259-282): nbytes (% 32 == 0) int8 values
 * (b & 63) - 32 from keyed BLAKE3 random_hash(block, label, key, prepend=0). If zero_me != NULL its
 * first zero_n int32 words are set to 0 (per-call counters, no extra memset launch). */
int uwc_noise_uniform(int8_t* out, uint64_t nbytes, const uint32_t* label, const uint32_t* key, int32_t* zero_me,
                      int zero_n, void* stream);

/* Replaces ops.noise_perm (ops.py:128-131, kernels.cu:284-301): k packed pairs
 * first | second << 16, first = u & (r-1), second = first ^ (1 + mulhi(r-1, u)); r a power of two. */
int uwc_noise_perm(uint32_t* out, uint32_t k, uint32_t r, const uint32_t* label, const uint32_t* key, void* stream);

/* Replaces ops.noise_rows (ops.py:134-142, kernels.cu:303-372). For each of `rows` rows of src
 * (rows x k int8): dst = src + E[first] - E[second] under Pn (if dst); projection under Pp written
 * as lmax balanced base-128 limbs to corr[li][row][corr_off + j] (row stride 2r) and max |proj|
 * folded into *maxabs with atomicMax (if Pp); E copied to corr[li][row][ecopy_off + j] (if
 * ecopy_off >= 0). rows % 8 == 0, k % 16 == 0, r in {64,128,256}. */
int uwc_noise_rows(const int8_t* src, int rows, int k, int r, const int8_t* E, const uint32_t* Pn, int8_t* dst,
                   const uint32_t* Pp, int8_t* corr, int corr_off, int ecopy_off, int32_t* maxabs, int lmax,
                   void* stream);

/* Replaces ops.proj_matrix (ops.py:152-158, kernels.cu:397-404): S^T (r x k int8),
 * S^T[j][l] = [P.first(l) == j] - [P.second(l) == j]. */
int uwc_proj_matrix(const uint32_t* P, int k, int r, int8_t* St, void* stream);

/* Replaces the tail of ops.project (ops.py:161-168, kernels.cu:374-395): balanced base-128
 * limbs of an int32 projection (rows x r) into corr[li][row][corr_off + j], max |proj| into *maxabs. */
int uwc_proj_corr(const int32_t* proj, int rows, int r, int8_t* corr, int corr_off, int32_t* maxabs, int lmax,
                  void* stream);

/* ---- the NoisyGEMM ----------------------------------------------------------------------
 * Replaces ops.gemm (ops.py:185-198) / kernel noisy_gemm (kernels.cu:482-715), on tcgen05
 * kind::i8 tensor cores with TMEM accumulators.
 * C = A B^T, A: m x k, B: n x k, int8, k contiguous (row stride k bytes, 16-byte aligned).
 *  flags & UWC_FLAG_HASH   : every r columns of k, XOR-fold each 8x16 hash tile (rows g+8i,
 *                            cols 2t+{0,1}+8j of a 64x64 block) into msg[c % 16] (rotl 13);
 *                            at the end hash = BLAKE3_keyed(key, msg) and, if hash <= target
 *                            (LE U256), append {row_off, col_off, hash[8]} to wins
 *                            (wins[0] = count, then max_wins records of UWC_WIN_WORDS words;
 *                            the count keeps counting past max_wins). m % 64 == 0, n % 64 == 0,
 *                            r in {64, 128, 256}, k % r == 0.
 *  flags & UWC_FLAG_DENOISE: subtract sum_li 128^li corrA[li] corrB[li]^T (K' = 2r per limb)
 *                            with L limbs chosen from max(maxabs[0], maxabs[1]) (<= lmax).
 *  out_mode                : UWC_OUT_NONE / UWC_OUT_I32 (int32 m x n) / UWC_OUT_BF16
 *                            (RNE of (float(acc) * a_scale[i]) * b_scale[j]) / UWC_OUT_F32
 *                            (same expression in fp32, the detrt dequant).
 * Without flags any m >= 1 works (rows past m are read as zero and not stored); k % 16 == 0.
 * workspace: device memory of at least uwc_gemm_workspace_bytes(m, n, flags, out_mode) bytes,
 *            16-byte aligned, any contents; unused (may be NULL) when that size is 0. Hashed calls
 *            without an output need none (the tile messages live in shared memory). A hashed call
 *            with an output runs as one kernel and stages each unit's raw int32 product there
 *            (256 KiB per SM) until the unit's tile hashes and correction are done; a plain
 *            split-K call with an F32 / BF16 output and m > 64 sums its int32 partials there
 *            (m * n * 4 bytes); plain calls with m <= 64 run the weight-streaming GEMM below and
 *            need none. Calls that overlap on the GPU must not share a workspace. */
uint64_t uwc_gemm_workspace_bytes(int m, int n, int flags, int out_mode);
int uwc_gemm(const int8_t* A, const int8_t* B, int m, int n, int k, int r, int flags, const int8_t* corrA,
             const int8_t* corrB, const int32_t* maxabs, int lmax, const uint32_t* key, const uint32_t* target,
             uint32_t* wins, int max_wins, const float* a_scale, const float* b_scale, void* out, int out_mode,
             void* workspace, uint64_t workspace_bytes, void* stream);

/* ---- the weight-streaming GEMM (decode-sized m) -------------------------------------------
 * New (the reference has no small-m path): out = X W^T for X m x k (1 <= m <= 64), W n x k, int8,
 * k contiguous, k % 16 == 0, X and W 16-byte aligned. W is read from HBM once: 128-row blocks of W
 * on the tensor core's M side, X on its N side, k split over a thread-block cluster whose CTAs add
 * their partial tiles in distributed shared memory. No workspace, no memset, one launch. The
 * epilogue `epi`:
 *   UWC_SEPI_I32     int32 out (m x n)                               (DetLinear.int_gemm)
 *   UWC_SEPI_F32     fmul(fmul(float(acc), x_scale[i]), w_scale[j])   (qwen3.py:125)
 *   UWC_SEPI_BF16    the same rounded to bf16 (RNE)
 *   UWC_SEPI_RESID   fadd(resid[i][j], the F32 value), resid m x n fp32 (NULL: the F32 value)
 *                    (detgpu kernels.py:346-354, the row-parallel output + residual)
 *   UWC_SEPI_SWIGLU  W = [gate; up], I = n / 2 rows each (n % 128 == 0); out m x I fp32 =
 *                    fmul(det_silu(g), u) of the dequantized pair (gate row f, up row I + f;
 *                    w_scale in the same order), detgpu kernels.py:356-396.
 * epi | UWC_SEPI_EARLY_W: W is not written by the kernel launched just before this call on the
 * stream (static weights), so the call may start streaming W while that kernel finishes.
 * uwc_gemm takes this path by itself for plain calls with m <= 64 (without UWC_SEPI_EARLY_W). */
#define UWC_SEPI_I32 0
#define UWC_SEPI_F32 1
#define UWC_SEPI_BF16 2
#define UWC_SEPI_RESID 3
#define UWC_SEPI_SWIGLU 4
#define UWC_SEPI_EARLY_W 0x100
int uwc_gemm_stream(const int8_t* X, const int8_t* W, int m, int n, int k, const float* x_scale,
                    const float* w_scale, const float* resid, void* out, int epi, void* stream);
/* The same epilogues at any m (replaces the int32 product + dequant_residual / swiglu passes of
 * runtime/detgpu/stages.py:117-153 with one kernel): m <= 64 runs uwc_gemm_stream, larger m the
 * tcgen05 GEMM with the output step in its epilogue (SWIGLU: each 256-row B tile is 128 gate rows
 * over their 128 up rows; n % 8 == 0). workspace: uwc_gemm_epi_workspace_bytes(m, n, epi) bytes
 * (a skinny split-K call's int32 sum; 0 otherwise), 16-byte aligned. */
uint64_t uwc_gemm_epi_workspace_bytes(int m, int n, int epi);
int uwc_gemm_epi(const int8_t* A, const int8_t* W, int m, int n, int k, const float* a_scale, const float* w_scale,
                 const float* resid, void* out, int epi, void* workspace, uint64_t workspace_bytes, void* stream);

/* ---- tensor-parallel decode over NVLink peer memory ---------------------------------------
 * New (the reference splits models only into pipeline stages, runtime/detrt/qwen3.py:151-158).
 * Each rank allocates one exchange buffer (uwc_tp_alloc, zero-filled, same max_m / max_n on every
 * rank), passes its IPC handle to the others (uwc_ipc_handle, UWC_IPC_HANDLE_BYTES bytes, sent by
 * the caller's own transport) and maps theirs (uwc_ipc_open). A UwcTP names this rank and every
 * rank's buffer as mapped here (base[rank] = its own). Every rank must make the same sequence of
 * uwc_*_tp calls on its buffer, each on its own GPU; a call waits (bounded, UWC_DEV_TIMEOUT) for
 * the peers' contributions to the same call. Values cross NVLink as 8-byte words tagged with the
 * call's epoch (a device-side call counter), which the receiver polls: no flags or fences. The wait
 * bound is 10 s (ranks may reach a call seconds apart at start-up); UWC_HOOK_WAIT_NS overrides it.
 *   uwc_quant_act_tp    uwc_quant_act of a row-parallel input shard with the absmax of the whole
 *                       row: each rank's shard absmax goes to every peer, each takes the maximum
 *                       (the fwht_absmax + MAX all-reduce + quant_act_global sequence, in one kernel);
 *                       m <= max_m.
 *   uwc_gemm_stream_tp  uwc_gemm_stream whose int32 product is summed over the ranks before the
 *                       epilogue (the row-parallel GEMM + SUM all-reduce + dequant/residual, in
 *                       one kernel): with fewer than 8 ranks each rank's partial slices go to every
 *                       peer and each rank adds them in rank order; from 8 ranks on each slice's
 *                       owner rank adds them and sends the sum to every rank. m <= max_m, n <= max_n,
 *                       epi UWC_SEPI_I32 / F32 / BF16 / RESID (| UWC_SEPI_EARLY_W). */
#define UWC_TP_MAX_WORLD 8
#define UWC_IPC_HANDLE_BYTES 64
typedef struct UwcTP {
  int rank, world, max_m, max_n;
  void* base[UWC_TP_MAX_WORLD];
} UwcTP;
uint64_t uwc_tp_buffer_bytes(int max_m, int max_n);
int uwc_tp_alloc(int max_m, int max_n, void** buf);
int uwc_tp_free(void* buf);
int uwc_ipc_handle(const void* buf, void* handle);
int uwc_ipc_open(const void* handle, void** peer_buf);
int uwc_ipc_close(void* peer_buf);
int uwc_quant_act_tp(const float* x, int m, int k, int bs, int8_t* q, float* scale, const UwcTP* tp, void* stream);
/* A device-side barrier of the ranks over the same exchange (one more call in the sequence): the
 * ranks' streams leave it within about one NVLink write latency of each other. */
int uwc_tp_barrier(const UwcTP* tp, void* stream);
int uwc_gemm_stream_tp(const int8_t* X, const int8_t* W, int m, int n, int k, const float* x_scale,
                       const float* w_scale, const float* resid, void* out, int epi, const UwcTP* tp, void* stream);

/* ---- a mined weight: the per-block and per-call sequences as single calls --------------------
 * MinedWeight (miner/ampere/uwc_ampere/ops.py:205-371) keeps its state in two caller-owned device
 * buffers whose layouts are fixed functions of the shapes:
 *   block      everything derived from B^T (n x k) and the block key, written by
 *              uwc_mined_setup_block and only read by the per-call functions;
 *   workspace  everything a call derives from A (m x k); every call overwrites it, so calls that
 *              overlap on the GPU need workspaces of their own (the reference shares one workspace
 *              per (device, m, k, r) among the layers of a model, ops.py:258-277: so can callers).
 * The *_layout functions write the byte offset of each part (the UWC_MB_* / UWC_MW_* indices) and,
 * at index UWC_MB_BYTES / UWC_MW_BYTES, the total size. Shapes: n % 64 == 0, k % 64 == 0,
 * r in {64, 128, 256}, k % r == 0, k <= 65536; m % 64 == 0 for the per-call functions. */
#define UWC_MB_CONSTS 0 /* 64 u32: job key, b_seed, target, noise labels A/B, seed salts A/B */
#define UWC_MB_EBRT 1   /* n x r int8: B-side noise factor */
#define UWC_MB_PB 2     /* k u32: B-side noise permutation, first | second << 16 */
#define UWC_MB_SBT 3    /* r x k int8: projection matrix of P_B */
#define UWC_MB_BPEBT 4  /* n x k int8: the noised weight B + F */
#define UWC_MB_BYTES 5
#define UWC_MW_A_SEED 0 /* 8 u32: the call's a_seed (the tile-hash key) */
#define UWC_MW_MAXABS 1 /* 2 int32: max |X|, max |Y| (forward) */
#define UWC_MW_EAL 2    /* m x r int8 */
#define UWC_MW_PA 3     /* k u32 */
#define UWC_MW_APEA 4   /* m x k int8: the noised A + E */
#define UWC_MW_B3 5     /* commitment scratch */
#define UWC_MW_GEMM 6   /* the hashed GEMM's workspace (uwc_gemm_workspace_bytes) */
#define UWC_MW_SAT 7    /* forward: r x k int8 projection matrix of P_A */
#define UWC_MW_CORRA 8  /* forward: L x m x 2r int8, [X_li | EAL] */
#define UWC_MW_CORRB 9  /* forward: L x n x 2r int8, [EBRt | Y_li] */
#define UWC_MW_PROJA 10 /* forward: m x r int32 */
#define UWC_MW_PROJB 11 /* forward: n x r int32 */
#define UWC_MW_BYTES 12
/* offsets: UWC_MB_BYTES + 1 entries. */
int uwc_mined_block_layout(int n, int k, int r, uint64_t* offsets);
/* offsets: UWC_MW_BYTES + 1 entries. forward = 0: the layout uwc_mine_attempt needs; 1: the one of
 * uwc_mined_forward with the given hash flag and out_mode (the forward parts are sized 0 otherwise). */
int uwc_mined_workspace_layout(int m, int n, int k, int r, int forward, int hash, int out_mode, uint64_t* offsets);
/* MinedWeight.setup_block (ops.py:233-253): commit to Bt (device, n x k int8, values in [-64, 64])
 * under the 32-byte job key, b_seed = BLAKE3(job_key || BLAKE3_keyed(salt_B, root_B || n)), the
 * B-side noise EBRt and P_B, BpEBt = Bt + EBRt P_B and the projection matrix of P_B, into `block`.
 * job_key (32 bytes) and target (8 LE words of the 256-bit tile target) are HOST memory, copied in
 * with cudaMemcpyAsync (so this call cannot be captured in a graph; the per-call ones can).
 * scratch: device memory of at least 4 * uwc_b3_scratch_words(n * k) bytes. */
int uwc_mined_setup_block(const int8_t* Bt, int n, int k, int r, const uint8_t* job_key, const uint32_t* target,
                          void* block, uint64_t block_bytes, void* scratch, uint64_t scratch_bytes, void* stream);
/* MinedWeight.noise_mine (ops.py:349-364): one mining attempt on the nonce matrix A (device, m x k
 * int8): a_seed = BLAKE3(b_seed || BLAKE3_keyed(salt_A, root_A || m)), A-side noise, ApEA, then the
 * hashed GEMM ApEA BpEBt^T with every 8 x 16 tile hashed and compared to the block's target; win
 * records into wins (count zeroed by this call, see uwc_gemm). No output matrix, no projections. */
int uwc_mine_attempt(const int8_t* A, int m, int n, int k, int r, const void* block, uint32_t* wins, int max_wins,
                     void* workspace, uint64_t workspace_bytes, void* stream);
/* MinedWeight.forward (ops.py:281-347): the mining attempt's preparation, the rank-r projections
 * X = A P_B^T and Y = BpEBt P_A^T as balanced base-128 limbs (ops.py:152-168, on the tensor cores:
 * the reference's UWC_PROJ_GEMM path), then the GEMM with
 * FLAG_DENOISE (and FLAG_HASH when hash != 0): out = A Bt^T exactly, in out_mode (I32, BF16, F32
 * with a_scale (m) and b_scale (n) as in uwc_gemm). The winning tiles equal uwc_mine_attempt's. */
int uwc_mined_forward(const int8_t* A, int m, int n, int k, int r, const float* a_scale, const float* b_scale,
                      const void* block, int hash, uint32_t* wins, int max_wins, void* out, int out_mode,
                      void* workspace, uint64_t workspace_bytes, void* stream);

/* ---- measurement --------------------------------------------------------------------------
 * The tensor core's int8 rate on the current device (no reference counterpart: a roofline
 * denominator). uwc_peak_i8 launches one CTA per SM, each issuing iters x 8 back-to-back
 * tcgen05.mma kind::i8 (M 128, N 256, K 32) from fixed shared-memory tiles into two TMEM
 * accumulators; time it with events on `stream`. uwc_peak_i8_ops(iters): its int8 operations
 * (2 per multiply-add). iters in [1, 131072]. */
int uwc_peak_i8(int iters, void* stream);
double uwc_peak_i8_ops(int iters);

/* ---------------------------------------------------------------- deterministic linear: producers
 * and consumers of the int8 GEMM, bit-identical to runtime/detrt's emulated-fp32 ops (every + - * /
 * sqrt rounded once, detrt's order; exact maxima; int64 fixed-point sums). One CTA per row; rows of
 * up to 51200 values. bs: Hadamard block size, 0/1 = none, else a power of two dividing k.
 * Pointers to device memory; x rows 16-byte aligned, q rows 4-byte aligned, k % 4 == 0. */

/* detrt.core.quant_act (runtime/detrt/core.py:188-196; GPU form runtime/detgpu/kernels.py:75-115):
 * y = fwht(x, bs), s = max(max|y|, 1e-8) / 64, q = clamp(rint(y / s), -64, 64) (int8 m x k),
 * scale = s * (1 / sqrt(bs)) when bs > 1 else s (float32 m). */
int uwc_quant_act(const float* x, int m, int k, int bs, int8_t* q, float* scale, void* stream);
/* The same from bf16 rows: ops.quant_rows_had (miner/ampere/uwc_ampere/ops.py:172-181, kernels.cu:723-778). */
int uwc_quant_rows_had(const uint16_t* x_bf16, int m, int k, int bs, int8_t* q, float* scale, void* stream);
/* quant_act split for a row-parallel (column-sharded) linear; no counterpart in the reference,
 * which has no tensor parallelism. fwht_absmax: amax[i] = max|fwht(x_i, bs)| of this shard.
 * quant_act_global: quant_act of this shard with the row absmax amax[i] given (the max over all
 * shards, e.g. after an all-reduce MAX): identical q and scale to quant_act on the full row. */
int uwc_fwht_absmax(const float* x, int m, int k, int bs, float* amax, void* stream);
int uwc_quant_act_global(const float* x, int m, int k, int bs, const float* amax, int8_t* q, float* scale,
                         void* stream);
/* quant_act(det_rmsnorm(x, w, eps), bs) (runtime/detgpu/kernels.py:117-191, 712-728): the
 * normalized row stays on chip. eps is rounded to float32 as detrt does. */
int uwc_rmsnorm_quant(const float* x, const float* w, int m, int k, int bs, double eps, int8_t* q, float* scale,
                      void* stream);
/* quant_act(det_silu(g) * u, bs) with [g | u] = fmul(fmul(float(acc), s3[i]), sw[j]) of the gate/up
 * GEMM output acc (int32 m x 2I) (runtime/detgpu/kernels.py:356-396, 816-826); q: int8 m x I. */
int uwc_swiglu_quant(const int32_t* acc, const float* s3, const float* sw, int m, int I, int bs, int8_t* q,
                     float* scale, void* stream);
/* h = fmul(det_silu(g), u) as fp32 (m x I): the input of a row-parallel down projection, which
 * quantizes its own column shard (uwc_fwht_absmax / uwc_quant_act_global). No counterpart in the
 * reference (it has no tensor parallelism); same per-element ops as uwc_swiglu_quant. m <= 65535. */
int uwc_swiglu(const int32_t* acc, const float* s3, const float* sw, int m, int I, float* h, void* stream);
/* out = x + fmul(fmul(float(acc), s[i]), sw[j]) (runtime/detgpu/kernels.py:346-354, 805-813);
 * x may be NULL: out = fmul(fmul(float(acc), s[i]), sw[j]), the plain dequant. */
int uwc_dequant_residual(const int32_t* acc, const float* s, const float* sw, const float* x, int m, int k,
                         float* out, void* stream);
/* The qkv GEMM output (int32 N x (H + 2 Hkv) * 128) -> int8 q (N,H,128), k, v (N,Hkv,128) with
 * per-head float32 scales (runtime/detgpu/kernels.py:303-344, 788-802): dequant, q/k head RMSNorm
 * when qknorm (Qwen3), rope with cos_t / sin_t rows (row r uses position r % T), quant_sym(127). */
int uwc_qkv_post(const int32_t* acc, const float* s1, const float* sw, const float* qnw, const float* knw,
                 const float* cos_t, const float* sin_t, int N, int T, int H, int Hkv, double eps, int qknorm,
                 int8_t* qq, float* qs, int8_t* kq, float* ks, int8_t* vq, float* vs, void* stream);
/* uwc_qkv_post with full cos / sin tables and the start position in device memory: row r uses
 * rope position *pos + r % T (a decode step's graph reads the position instead of baking it in). */
int uwc_qkv_post_at(const int32_t* acc, const float* s1, const float* sw, const float* qnw, const float* knw,
                    const float* cos_table, const float* sin_table, const int* pos, int N, int T, int H, int Hkv,
                    double eps, int qknorm, int8_t* qq, float* qs, int8_t* kq, float* ks, int8_t* vq, float* vs,
                    void* stream);
/* uwc_qkv_post_at with the keys and values written straight into a KV cache (the qkv_post +
 * kv_append pair of a decode step as one kernel): token r % T of sequence r / T lands at cache
 * position *pos + r % T of kc / vc ((B, Hkv, maxlen, 128) int8) and skc / svc ((B, Hkv, maxlen)
 * scales); positions >= maxlen are not written. Same values as uwc_qkv_post_at + uwc_kv_append. */
int uwc_qkv_post_kv(const int32_t* acc, const float* s1, const float* sw, const float* qnw, const float* knw,
                    const float* cos_table, const float* sin_table, const int* pos, int N, int T, int H, int Hkv,
                    double eps, int qknorm, int8_t* qq, float* qs, int8_t* kc, float* skc, int8_t* vc, float* svc,
                    int maxlen, void* stream);

/* Deterministic attention from quantized q, k, v (runtime/detrt/qwen3.py:254-283 _attention;
 * GPU form runtime/detgpu/kernels.py:731-771 attention): exact int32 Q K^T, scores
 * fmul(fmul(fmul(float(dot), qs), ks), inv_sqrt_hd), causal mask, det_exp, exact int64 row sum,
 * P * sv quantized to 14 bits, P V as two 7-bit limbs summed exactly, times the row scale.
 * Queries qq (B * Tq, H, 128) int8 and qs (B * Tq, H) are the Tq new tokens of each of B sequences
 * at absolute positions start .. start + Tq - 1; query t sees keys 0 .. start + t. Keys / values
 * (int8, 128 per head) are read at kc + b * kv_seq + j * kv_tok + g * kv_head (element strides,
 * multiples of 16), their scales at ks + b * s_seq + j * s_tok + g * s_head; g = h / (H / Hkv).
 * Token-major prefill (the detgpu call): kv_seq = Tq * Hkv * 128, kv_tok = Hkv * 128,
 * kv_head = 128; a KV cache (B, Hkv, maxlen, 128): kv_seq = Hkv * maxlen * 128, kv_head =
 * maxlen * 128, kv_tok = 128. out (B * Tq, H * 128) float32. UWC_ERR_SHAPE when one query row's
 * start + Tq scores do not fit in shared memory (about 51 000 keys). */
int uwc_attention(const int8_t* qq, const float* qs, const int8_t* kc, const float* ks, const int8_t* vc,
                  const float* vs, int B, int Tq, int start, int H, int Hkv, long long kv_seq, long long kv_tok,
                  long long kv_head, long long s_seq, long long s_tok, long long s_head, float inv_sqrt_hd,
                  float* out, void* stream);
/* uwc_attention for many query rows on the tensor cores: S = Q K^T and O = [P_hi; P_lo] V as
 * batched tcgen05 int8 GEMMs (uwc_gemm_batched), the scale chain and softmax per query row between
 * them; the same bits as uwc_attention (exact integer sums). Same arguments plus a device
 * workspace of uwc_attention_tc_workspace_bytes(B, Tq, start, H, Hkv) bytes (16-byte aligned).
 * start + Tq <= 131072 (the P V limb sums stay below 2^31) and 4 (start + Tq) floats of shared
 * memory per query row. Replaces the same call as uwc_attention (runtime/detgpu/kernels.py
 * attention, the prefill form). */
uint64_t uwc_attention_tc_workspace_bytes(int B, int Tq, int start, int H, int Hkv);
int uwc_attention_tc(const int8_t* qq, const float* qs, const int8_t* kc, const float* ks, const int8_t* vc,
                     const float* vs, int B, int Tq, int start, int H, int Hkv, long long kv_seq, long long kv_tok,
                     long long kv_head, long long s_seq, long long s_tok, long long s_head, float inv_sqrt_hd,
                     float* out, void* workspace, uint64_t workspace_bytes, void* stream);
/* Batched exact int8 GEMM, int32 out: out[bt] (m x n, contiguous per batch) = A[bt] B[bt / b_bdiv]^T
 * for bt < nbatch, A[bt] the m x k rows from row bt * a_brows of A, B[g] the n x k rows from row
 * g * b_brows of B (both k-contiguous, row length k; k % 16 == 0, n % 4 == 0). causal 1 computes
 * only the 128 x 256 output blocks some row sees (row t sees columns j <= cshift + t); causal 2
 * stops a 128-row block's k range after column cshift + (m0 % qrows) + 127 (A stacks two qrows-row
 * halves). No counterpart in the reference (its attention is SIMT, runtime/detgpu/kernels.py). */
int uwc_gemm_batched(const int8_t* A, const int8_t* B, int m, int n, int k, int nbatch, long long a_brows,
                     long long b_brows, int b_bdiv, int causal, int cshift, int qrows, int32_t* out, void* stream);
/* uwc_attention with the start position read from device memory (*start <= max_start), so one
 * CUDA graph serves every decode step; shared memory is sized for max_start + Tq keys. No
 * counterpart in the reference (its decode runs eagerly, runtime/detrt/qwen3.py:315-329). */
int uwc_attention_at(const int8_t* qq, const float* qs, const int8_t* kc, const float* ks, const int8_t* vc,
                     const float* vs, int B, int Tq, const int* start, int max_start, int H, int Hkv,
                     long long kv_seq, long long kv_tok, long long kv_head, long long s_seq, long long s_tok,
                     long long s_head, float inv_sqrt_hd, float* out, void* stream);
/* The KV cache write of runtime/detrt/qwen3.py:249-252: token t of sequence b (kq / vq (B*T, Hkv,
 * 128) int8, ks / vs (B*T, Hkv) float32) into a cache k, v (B, Hkv, maxlen, 128), sk, sv
 * (B, Hkv, maxlen) at position *pos + t (device memory; positions past maxlen are skipped). */
int uwc_kv_append(const int8_t* kq, const float* ks, const int8_t* vq, const float* vs, int B, int T, int Hkv,
                  int maxlen, const int* pos, int8_t* kc, float* skc, int8_t* vc, float* svc, void* stream);
/* det_rmsnorm (runtime/detrt/core.py:151-159) of m rows of k floats: the final norm of
 * DetQwen3.forward (runtime/detrt/qwen3.py:299), float32 out. */
int uwc_rmsnorm(const float* x, const float* w, int m, int k, double eps, float* out, void* stream);
/* DetQwen3.logprobs (runtime/detrt/qwen3.py:302-312) of m rows of V logits: z = lg - max,
 * lp = z - det_log(exact_rowsum(det_exp(z), 2^18)) into lp (may be NULL), and the greedy token
 * of generate_greedy (qwen3.py:323, the first index of the maximal lp) into tok (may be NULL). */
int uwc_logprobs(const float* logits, int m, int V, float* lp, long long* tok, void* stream);

/* Stage-output commitments (runtime/detgpu/sha.py; formats runtime/detrt/stage.py:26-72 and
 * runtime/agent/proto.py:24-35): for float32 rows of D values, row_root = RFC 6962 Merkle root of
 * sha256(0x00 || block) over 1 KiB blocks of the row's little-endian bytes, the token leaf
 * sha256(0x00 || "sout" || u32le t || row_root) with t = row % T, and a stage's root = the Merkle
 * root of its T leaves. Digests are written as 8 big-endian SHA-256 state words. D <= 8192.
 * Scratch: uwc_stage_scratch_words(nrows, D) u32 words of caller device memory. */
uint64_t uwc_stage_scratch_words(long long nrows, int D);
/* The token leaves of nrows rows (nrows a multiple of T) into leaves (nrows x 8 words):
 * sout_leaves (runtime/detgpu/sha.py:103-135). */
int uwc_stage_out_leaves(const float* rows, long long nrows, int D, int T, uint32_t* scratch,
                         uint64_t scratch_words, uint32_t* leaves, void* stream);
/* The roots of B stages of T rows each (rows B*T x D) into roots (B x 8 words): stage_roots_gpu
 * (runtime/detgpu/sha.py:138-163), agent.proto.stage_output_root per stage. */
int uwc_stage_roots(const float* rows, int B, int T, int D, uint32_t* scratch, uint64_t scratch_words,
                    uint32_t* roots, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* UWC_B200_H */
