// A mined weight's two sequences behind one C call each: the per-block preparation of B^T
// (MinedWeight.setup_block, miner/ampere/uwc_ampere/ops.py:233-253) and the per-call work on a
// nonce matrix A, either a pure mining attempt (MinedWeight.noise_mine, ops.py:349-364) or the
// hashed, exactly denoised forward (MinedWeight.forward, ops.py:281-347).
//
// The caller owns two device buffers: the block (everything derived from B^T and the block key,
// written once by uwc_mined_setup_block and only read afterwards) and a workspace (everything a
// call derives from A, overwritten by every call). Their layouts are fixed functions of the shapes
// (uwc_mined_block_layout / uwc_mined_workspace_layout), so a host binding can view the parts.
// Nothing here allocates, synchronizes or copies to the host; every launch goes to the caller's
// stream. The order of the steps is the protocol's: commit to the operand, derive its seed, then
// its noise, then the noised operand (and for a forward the rank-r projections of the exact
// denoise), then the hashed GEMM.
#include <cstring>

#include "uwc_device.cuh"
#include "uwc_host.h"

namespace {

constexpr uint64_t kAlign = 256;
constexpr uint64_t up(uint64_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

// Word offsets inside the block's constants region (64 u32 words).
enum : int { C_JOB_KEY = 0, C_B_SEED = 8, C_TARGET = 16, C_LABEL_A = 24, C_LABEL_B = 32, C_SALT_A = 40, C_SALT_B = 48 };

// Pearl cert-v3 constants (miner/ampere/uwc_ampere/reference.py:22-25): the noise labels are the
// ASCII tensor names zero-padded to 32 bytes; the seed salts are BLAKE3("pearl/cert-v3/noise-seed/A")
// and BLAKE3(".../B"), as little-endian words.
const char kLabelA[] = "A_tensor";
const char kLabelB[] = "B_tensor";
const uint8_t kSaltA[32] = {0x82, 0x49, 0x40, 0x6c, 0xa0, 0xed, 0x15, 0x16, 0x96, 0x16, 0xf6, 0x92, 0xfc, 0xf0, 0x76, 0xf8,
                            0x92, 0xdb, 0xdb, 0x2a, 0x70, 0x23, 0xb8, 0x52, 0xf0, 0xd4, 0x77, 0x19, 0xc3, 0x90, 0x01, 0x7b};
const uint8_t kSaltB[32] = {0x11, 0x30, 0x06, 0x32, 0xec, 0x63, 0x01, 0xca, 0x2b, 0xe2, 0xaf, 0x71, 0x8b, 0x3f, 0x4d, 0x4f,
                            0x1a, 0xe9, 0xc6, 0x39, 0x88, 0xe8, 0xcc, 0x04, 0x48, 0x44, 0x30, 0x1d, 0x71, 0xb8, 0x9a, 0xa9};

// Limbs that always cover a projection of k values in [-127, 127] (ops.py:18-24).
int limbs_for(int k) {
  const int64_t bound = 127LL * k;
  int64_t cap = 63;
  int L = 1;
  while (cap < bound) {
    L++;
    cap = cap * 128 + 63;
  }
  return L;
}

bool shapes_ok(int n, int k, int r) {
  return n > 0 && k > 0 && n % 64 == 0 && k % 64 == 0 && (r == 64 || r == 128 || r == 256) && k % r == 0 &&
         k <= 65536;
}

void block_layout(int n, int k, int r, uint64_t* off) {
  uint64_t o = 0;
  off[UWC_MB_CONSTS] = o; o += up(64 * 4);
  off[UWC_MB_EBRT] = o;   o += up((uint64_t)n * r);
  off[UWC_MB_PB] = o;     o += up((uint64_t)k * 4);
  off[UWC_MB_SBT] = o;    o += up((uint64_t)r * k);
  off[UWC_MB_BPEBT] = o;  o += up((uint64_t)n * k);
  off[UWC_MB_BYTES] = o;
}

void workspace_layout(int m, int n, int k, int r, int forward, int hash, int out_mode, uint64_t* off) {
  const int L = limbs_for(k);
  const int flags = (hash ? UWC_FLAG_HASH : 0) | (forward ? UWC_FLAG_DENOISE : 0);
  uint64_t o = 0;
  off[UWC_MW_A_SEED] = o; o += up(8 * 4);
  off[UWC_MW_MAXABS] = o; o += up(2 * 4);
  off[UWC_MW_EAL] = o;    o += up((uint64_t)m * r);
  off[UWC_MW_PA] = o;     o += up((uint64_t)k * 4);
  off[UWC_MW_APEA] = o;   o += up((uint64_t)m * k);
  off[UWC_MW_B3] = o;     o += up(uwc_b3_scratch_words((uint64_t)m * k) * 4);
  off[UWC_MW_GEMM] = o;   o += up(uwc_gemm_workspace_bytes(m, n, flags, forward ? out_mode : UWC_OUT_NONE));
  const bool f = forward != 0;
  off[UWC_MW_SAT] = o;    o += f ? up((uint64_t)r * k) : 0;
  off[UWC_MW_CORRA] = o;  o += f ? up((uint64_t)L * m * 2 * r) : 0;
  off[UWC_MW_CORRB] = o;  o += f ? up((uint64_t)L * n * 2 * r) : 0;
  off[UWC_MW_PROJA] = o;  o += f ? up((uint64_t)m * r * 4) : 0;
  off[UWC_MW_PROJB] = o;  o += f ? up((uint64_t)n * r * 4) : 0;
  off[UWC_MW_BYTES] = o;
}

#define UWC_TRY(call)                  \
  do {                                 \
    const int _rc = (call);            \
    if (_rc != UWC_OK) return _rc;     \
  } while (0)

template <typename T>
T* at(void* base, uint64_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}
template <typename T>
const T* at(const void* base, uint64_t off) {
  return reinterpret_cast<const T*>(static_cast<const uint8_t*>(base) + off);
}

// Commit to A under the block key (seed prefix b_seed, salt A) and derive its noise: a_seed, EAL,
// P_A, and ApEA = A + EAL P_A (with EAL copied into every correction limb when corrA is given).
// Zeroes the win counter and maxabs on the way (no separate memset launches).
int prepare_a(const int8_t* A, int m, int k, int r, const void* block, const uint64_t* bo, void* ws,
              const uint64_t* wo, uint32_t* wins, int32_t* maxabs, int8_t* corrA, int L, cudaStream_t st) {
  const uint32_t* c = at<uint32_t>(block, bo[UWC_MB_CONSTS]);
  uint32_t* a_seed = at<uint32_t>(ws, wo[UWC_MW_A_SEED]);
  UWC_TRY(uwc_b3_root_and_seed(A, (uint64_t)m * k, c + C_JOB_KEY, c + C_B_SEED, c + C_SALT_A, (uint32_t)m, nullptr,
                               a_seed, at<uint32_t>(ws, wo[UWC_MW_B3]), uwc_b3_scratch_words((uint64_t)m * k), st));
  int8_t* EAL = at<int8_t>(ws, wo[UWC_MW_EAL]);
  UWC_TRY(uwc_noise_uniform_zero2(EAL, (uint64_t)m * r, c + C_LABEL_A, a_seed, reinterpret_cast<int32_t*>(wins),
                                  wins ? 1 : 0, maxabs, maxabs ? 2 : 0, st));
  uint32_t* PA = at<uint32_t>(ws, wo[UWC_MW_PA]);
  UWC_TRY(uwc_noise_perm(PA, (uint32_t)k, (uint32_t)r, c + C_LABEL_A, a_seed, st));
  return uwc_noise_rows(A, m, k, r, EAL, PA, at<int8_t>(ws, wo[UWC_MW_APEA]), nullptr, corrA, -1, corrA ? r : -1,
                        nullptr, corrA ? L : 0, st);
}

}  // namespace

extern "C" int uwc_mined_block_layout(int n, int k, int r, uint64_t* offsets) {
  if (!offsets) return UWC_ERR_ARG;
  if (!shapes_ok(n, k, r)) return UWC_ERR_SHAPE;
  block_layout(n, k, r, offsets);
  return UWC_OK;
}

extern "C" int uwc_mined_workspace_layout(int m, int n, int k, int r, int forward, int hash, int out_mode,
                                          uint64_t* offsets) {
  if (!offsets || out_mode < 0 || out_mode > 3) return UWC_ERR_ARG;
  if (m <= 0 || m % 64 || !shapes_ok(n, k, r)) return UWC_ERR_SHAPE;
  workspace_layout(m, n, k, r, forward, hash, out_mode, offsets);
  return UWC_OK;
}

extern "C" int uwc_mined_setup_block(const int8_t* Bt, int n, int k, int r, const uint8_t* job_key,
                                     const uint32_t* target, void* block, uint64_t block_bytes, void* scratch,
                                     uint64_t scratch_bytes, void* stream) {
  if (!Bt || !job_key || !target || !block || !scratch) return UWC_ERR_ARG;
  if (!shapes_ok(n, k, r)) return UWC_ERR_SHAPE;
  if ((((uintptr_t)Bt) | ((uintptr_t)block) | ((uintptr_t)scratch)) & 15) return UWC_ERR_ALIGN;
  uint64_t bo[UWC_MB_BYTES + 1];
  block_layout(n, k, r, bo);
  if (block_bytes < bo[UWC_MB_BYTES]) return UWC_ERR_SCRATCH;
  const uint64_t b3_words = uwc_b3_scratch_words((uint64_t)n * k);
  if (scratch_bytes < b3_words * 4) return UWC_ERR_SCRATCH;
  UWC_CHECK_DEVICE();
  cudaStream_t st = (cudaStream_t)stream;
  // the constants: job key, (b_seed, written below), target, labels, salts. The copy from this
  // stack array is staged by the runtime before cudaMemcpyAsync returns (pageable source).
  uint32_t host[64];
  std::memset(host, 0, sizeof(host));
  std::memcpy(host + C_JOB_KEY, job_key, 32);
  std::memcpy(host + C_TARGET, target, 32);
  std::memcpy(host + C_LABEL_A, kLabelA, sizeof(kLabelA) - 1);
  std::memcpy(host + C_LABEL_B, kLabelB, sizeof(kLabelB) - 1);
  std::memcpy(host + C_SALT_A, kSaltA, 32);
  std::memcpy(host + C_SALT_B, kSaltB, 32);
  uint32_t* c = at<uint32_t>(block, bo[UWC_MB_CONSTS]);
  if (cudaMemcpyAsync(c, host, sizeof(host), cudaMemcpyHostToDevice, st) != cudaSuccess) {
    cudaGetLastError();
    return UWC_ERR_CUDA;
  }
  // b_seed = H(job_key || bind_b(root_B, n)) (ops.py:240-241)
  UWC_TRY(uwc_b3_root_and_seed(Bt, (uint64_t)n * k, c + C_JOB_KEY, c + C_JOB_KEY, c + C_SALT_B, (uint32_t)n, nullptr,
                               c + C_B_SEED, static_cast<uint32_t*>(scratch), b3_words, st));
  int8_t* EBRt = at<int8_t>(block, bo[UWC_MB_EBRT]);
  UWC_TRY(uwc_noise_uniform(EBRt, (uint64_t)n * r, c + C_LABEL_B, c + C_B_SEED, nullptr, 0, st));
  uint32_t* PB = at<uint32_t>(block, bo[UWC_MB_PB]);
  UWC_TRY(uwc_noise_perm(PB, (uint32_t)k, (uint32_t)r, c + C_LABEL_B, c + C_B_SEED, st));
  UWC_TRY(uwc_noise_rows(Bt, n, k, r, EBRt, PB, at<int8_t>(block, bo[UWC_MB_BPEBT]), nullptr, nullptr, -1, -1,
                         nullptr, 0, st));
  return uwc_proj_matrix(PB, k, r, at<int8_t>(block, bo[UWC_MB_SBT]), st);
}

extern "C" int uwc_mine_attempt(const int8_t* A, int m, int n, int k, int r, const void* block, uint32_t* wins,
                                int max_wins, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!A || !block || !wins || !workspace || max_wins < 0) return UWC_ERR_ARG;
  if (m <= 0 || m % 64 || !shapes_ok(n, k, r)) return UWC_ERR_SHAPE;
  if ((((uintptr_t)A) | ((uintptr_t)block) | ((uintptr_t)workspace)) & 15) return UWC_ERR_ALIGN;
  uint64_t bo[UWC_MB_BYTES + 1], wo[UWC_MW_BYTES + 1];
  block_layout(n, k, r, bo);
  workspace_layout(m, n, k, r, 0, 1, UWC_OUT_NONE, wo);
  if (workspace_bytes < wo[UWC_MW_BYTES]) return UWC_ERR_SCRATCH;
  UWC_CHECK_DEVICE();
  cudaStream_t st = (cudaStream_t)stream;
  UWC_TRY(prepare_a(A, m, k, r, block, bo, workspace, wo, wins, nullptr, nullptr, 0, st));
  const uint32_t* c = at<uint32_t>(block, bo[UWC_MB_CONSTS]);
  return uwc_gemm(at<int8_t>(workspace, wo[UWC_MW_APEA]), at<int8_t>(block, bo[UWC_MB_BPEBT]), m, n, k, r,
                  UWC_FLAG_HASH, nullptr, nullptr, nullptr, 0, at<uint32_t>(workspace, wo[UWC_MW_A_SEED]),
                  c + C_TARGET, wins, max_wins, nullptr, nullptr, nullptr, UWC_OUT_NONE,
                  at<void>(workspace, wo[UWC_MW_GEMM]), wo[UWC_MW_GEMM + 1] - wo[UWC_MW_GEMM], st);
}

extern "C" int uwc_mined_forward(const int8_t* A, int m, int n, int k, int r, const float* a_scale,
                                 const float* b_scale, const void* block, int hash, uint32_t* wins, int max_wins,
                                 void* out, int out_mode, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!A || !block || !workspace || (hash && (!wins || max_wins < 0))) return UWC_ERR_ARG;
  if (out_mode < 0 || out_mode > 3 || (out_mode != UWC_OUT_NONE && !out)) return UWC_ERR_ARG;
  if ((out_mode == UWC_OUT_BF16 || out_mode == UWC_OUT_F32) && (!a_scale || !b_scale)) return UWC_ERR_ARG;
  if (m <= 0 || m % 64 || !shapes_ok(n, k, r)) return UWC_ERR_SHAPE;
  if ((((uintptr_t)A) | ((uintptr_t)block) | ((uintptr_t)workspace) | ((uintptr_t)out)) & 15) return UWC_ERR_ALIGN;
  uint64_t bo[UWC_MB_BYTES + 1], wo[UWC_MW_BYTES + 1];
  block_layout(n, k, r, bo);
  workspace_layout(m, n, k, r, 1, hash, out_mode, wo);
  if (workspace_bytes < wo[UWC_MW_BYTES]) return UWC_ERR_SCRATCH;
  UWC_CHECK_DEVICE();
  cudaStream_t st = (cudaStream_t)stream;
  const int L = limbs_for(k);
  int32_t* maxabs = at<int32_t>(workspace, wo[UWC_MW_MAXABS]);
  int8_t* corrA = at<int8_t>(workspace, wo[UWC_MW_CORRA]);
  int8_t* corrB = at<int8_t>(workspace, wo[UWC_MW_CORRB]);
  // 1-3: a_seed, EAL, P_A, ApEA, EAL into every limb of corrA, maxabs and the win counter zeroed
  UWC_TRY(prepare_a(A, m, k, r, block, bo, workspace, wo, hash ? wins : nullptr, maxabs, corrA, L, st));
  // 4: X = A P_B^T as limbs beside EAL: [X_li | EAL] (ops.py:331-333), the sum on the tensor cores
  int32_t* projA = at<int32_t>(workspace, wo[UWC_MW_PROJA]);
  UWC_TRY(uwc_gemm(A, at<int8_t>(block, bo[UWC_MB_SBT]), m, r, k, 0, 0, nullptr, nullptr, nullptr, 0, nullptr, nullptr,
                   nullptr, 0, nullptr, nullptr, projA, UWC_OUT_I32, nullptr, 0, st));
  UWC_TRY(uwc_proj_corr(projA, m, r, corrA, 0, maxabs, L, st));
  // 5: Y = BpEBt P_A^T as limbs beside EBRt: [EBRt | Y_li]
  int8_t* SAt = at<int8_t>(workspace, wo[UWC_MW_SAT]);
  UWC_TRY(uwc_proj_matrix(at<uint32_t>(workspace, wo[UWC_MW_PA]), k, r, SAt, st));
  int32_t* projB = at<int32_t>(workspace, wo[UWC_MW_PROJB]);
  UWC_TRY(uwc_gemm(at<int8_t>(block, bo[UWC_MB_BPEBT]), SAt, n, r, k, 0, 0, nullptr, nullptr, nullptr, 0, nullptr,
                   nullptr, nullptr, 0, nullptr, nullptr, projB, UWC_OUT_I32, nullptr, 0, st));
  UWC_TRY(uwc_proj_corr_ecopy(projB, n, r, corrB, r, maxabs + 1, L, at<int8_t>(block, bo[UWC_MB_EBRT]), 0, st));
  // 6: the noisy GEMM: hash every tile (optional), subtract the correction exactly, scale
  const uint32_t* c = at<uint32_t>(block, bo[UWC_MB_CONSTS]);
  return uwc_gemm(at<int8_t>(workspace, wo[UWC_MW_APEA]), at<int8_t>(block, bo[UWC_MB_BPEBT]), m, n, k, r,
                  (hash ? UWC_FLAG_HASH : 0) | UWC_FLAG_DENOISE, corrA, corrB, maxabs, L,
                  at<uint32_t>(workspace, wo[UWC_MW_A_SEED]), c + C_TARGET, hash ? wins : nullptr, max_wins, a_scale,
                  b_scale, out, out_mode, at<void>(workspace, wo[UWC_MW_GEMM]),
                  wo[UWC_MW_GEMM + 1] - wo[UWC_MW_GEMM], st);
}
