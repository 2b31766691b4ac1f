/*
 * uwc_oracle.c -- CPU restatement of the cuPOW NoisyGEMM mining rules.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg may load it.
 * The product path (useful-work-coin_b200/) never links or calls it.
 *
 * What it restates (reference citations are paths inside srivassid/useful-work-coin):
 *   - BLAKE3 (published algorithm, blake3 spec; pinned against the PyPI `blake3` package,
 *     which is what miner/ampere/uwc_ampere/reference.py:15 uses).
 *   - keyed Merkle root of 1 KiB-padded bytes + the cert-v3 salted seed
 *     (miner/ampere/uwc_ampere/reference.py:33-64).
 *   - random_hash / uniform_matrix / perm_matrix (reference.py:67-93).
 *   - noise_rows: noising, rank-r projection, balanced base-128 limbs, maxabs
 *     (miner/ampere/uwc_ampere/kernels.cu:303-372, test oracle tests/test_kernels.py:133-156).
 *   - jackpot XOR-fold per hash tile and the keyed tile hash
 *     (reference.py:107-125,138-165; tile pattern pearl_glue.py:14-15).
 *   - exact int32 GEMM (the value noisy_gemm must produce after denoising, kernels.cu:598-673).
 *
 * Every function is plain C with fixed-width integers; threads (pthreads) only split
 * independent rows, so results do not depend on the thread count.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ BLAKE3 */
enum { B3_CHUNK_START = 1, B3_CHUNK_END = 2, B3_PARENT = 4, B3_ROOT = 8, B3_KEYED = 16 };

static const uint32_t B3_IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                                  0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
static const int B3_PERM[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};

static inline uint32_t ror32(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static inline void b3_g(uint32_t* s, int a, int b, int c, int d, uint32_t x, uint32_t y) {
  s[a] = s[a] + s[b] + x;
  s[d] = ror32(s[d] ^ s[a], 16);
  s[c] = s[c] + s[d];
  s[b] = ror32(s[b] ^ s[c], 12);
  s[a] = s[a] + s[b] + y;
  s[d] = ror32(s[d] ^ s[a], 8);
  s[c] = s[c] + s[d];
  s[b] = ror32(s[b] ^ s[c], 7);
}

/* BLAKE3 compression, truncated to the 8-word chaining value. */
void orc_b3_compress(const uint32_t cv[8], const uint32_t block[16], uint64_t counter,
                     uint32_t blen, uint32_t flags, uint32_t out[8]) {
  uint32_t s[16], m[16], t[16];
  for (int i = 0; i < 8; i++) s[i] = cv[i];
  for (int i = 0; i < 4; i++) s[8 + i] = B3_IV[i];
  s[12] = (uint32_t)counter;
  s[13] = (uint32_t)(counter >> 32);
  s[14] = blen;
  s[15] = flags;
  memcpy(m, block, sizeof(m));
  for (int r = 0; r < 7; r++) {
    b3_g(s, 0, 4, 8, 12, m[0], m[1]);
    b3_g(s, 1, 5, 9, 13, m[2], m[3]);
    b3_g(s, 2, 6, 10, 14, m[4], m[5]);
    b3_g(s, 3, 7, 11, 15, m[6], m[7]);
    b3_g(s, 0, 5, 10, 15, m[8], m[9]);
    b3_g(s, 1, 6, 11, 12, m[10], m[11]);
    b3_g(s, 2, 7, 8, 13, m[12], m[13]);
    b3_g(s, 3, 4, 9, 14, m[14], m[15]);
    for (int i = 0; i < 16; i++) t[i] = m[B3_PERM[i]];
    memcpy(m, t, sizeof(m));
  }
  for (int i = 0; i < 8; i++) out[i] = s[i] ^ s[i + 8];
}

static void load_words(const uint8_t* p, size_t n, uint32_t w[16]) {
  uint8_t buf[64];
  memset(buf, 0, 64);
  memcpy(buf, p, n);
  for (int i = 0; i < 16; i++)
    w[i] = (uint32_t)buf[4 * i] | ((uint32_t)buf[4 * i + 1] << 8) | ((uint32_t)buf[4 * i + 2] << 16) |
           ((uint32_t)buf[4 * i + 3] << 24);
}

/* Chaining value of chunk `idx` (len <= 1024 bytes); root=1 marks the single-chunk root. */
static void b3_chunk_cv(const uint8_t* p, size_t len, uint64_t idx, const uint32_t key[8], uint32_t kflag,
                        int root, uint32_t out[8]) {
  uint32_t cv[8], w[16];
  memcpy(cv, key, 32);
  size_t nblk = len == 0 ? 1 : (len + 63) / 64;
  for (size_t b = 0; b < nblk; b++) {
    size_t bl = (b + 1 == nblk) ? len - b * 64 : 64;
    load_words(p + b * 64, bl, w);
    uint32_t fl = kflag | (b == 0 ? B3_CHUNK_START : 0) | (b + 1 == nblk ? B3_CHUNK_END : 0) |
                  ((root && b + 1 == nblk) ? B3_ROOT : 0);
    orc_b3_compress(cv, w, idx, (uint32_t)bl, fl, cv);
  }
  memcpy(out, cv, 32);
}

/* BLAKE3 of `len` bytes; key==NULL -> unkeyed (IV), else keyed hash with the 8-word key.
 * The tree is merged level by level with the odd trailing node carried up, which is the same
 * left-balanced tree the spec's merge stack builds. */
void orc_b3_hash(const uint8_t* data, uint64_t len, const uint32_t* key, uint32_t out[8]) {
  uint32_t k8[8];
  uint32_t kflag = key ? B3_KEYED : 0;
  memcpy(k8, key ? key : B3_IV, 32);
  uint64_t nch = len == 0 ? 1 : (len + 1023) / 1024;
  if (nch == 1) {
    b3_chunk_cv(data, (size_t)len, 0, k8, kflag, 1, out);
    return;
  }
  uint32_t* cvs = (uint32_t*)malloc(nch * 32);
  for (uint64_t c = 0; c < nch; c++) {
    uint64_t cl = (c + 1 == nch) ? len - c * 1024 : 1024;
    b3_chunk_cv(data + c * 1024, (size_t)cl, c, k8, kflag, 0, cvs + 8 * c);
  }
  uint64_t cnt = nch;
  while (cnt > 1) {
    uint64_t pairs = cnt / 2;
    for (uint64_t i = 0; i < pairs; i++) {
      uint32_t blk[16];
      memcpy(blk, cvs + 16 * i, 64);
      uint32_t fl = B3_PARENT | kflag | (cnt == 2 ? B3_ROOT : 0);
      orc_b3_compress(k8, blk, 0, 64, fl, cvs + 8 * i);
    }
    if (cnt & 1) memmove(cvs + 8 * pairs, cvs + 8 * (cnt - 1), 32);
    cnt = pairs + (cnt & 1);
  }
  memcpy(out, cvs, 32);
  free(cvs);
}

/* Single-block keyed hash of a 64-byte message given as 16 LE words (key==NULL -> unkeyed). */
void orc_b3_hash64(const uint32_t* key, const uint32_t msg[16], uint32_t out[8]) {
  orc_b3_compress(key ? key : B3_IV, msg, 0, 64, B3_CHUNK_START | B3_CHUNK_END | B3_ROOT | (key ? B3_KEYED : 0),
                  out);
}

/* ------------------------------------------------------------------ seeds and noise */
/* v3 salted seed: seed = H(prefix || keyed(salt, root || dim_le32 || 0^28)) (reference.py:46-61). */
void orc_salted_seed(const uint32_t root[8], uint32_t dim, const uint32_t salt[8], const uint32_t prefix[8],
                     uint32_t seed[8]) {
  uint32_t msg[16], bound[8];
  memcpy(msg, root, 32);
  memset(msg + 8, 0, 32);
  msg[8] = dim;
  orc_b3_hash64(salt, msg, bound);
  memcpy(msg, prefix, 32);
  memcpy(msg + 8, bound, 32);
  orc_b3_hash64(NULL, msg, seed);
}

/* get_random_hash(index, label, key, prepend) (reference.py:67-71). */
void orc_random_hash(uint32_t index, const uint32_t label[8], const uint32_t key[8], int prepend, uint32_t out[8]) {
  uint32_t msg[16];
  memset(msg, 0, 32);
  memcpy(msg + 8, label, 32);
  msg[prepend] = 1u + index;
  orc_b3_hash64(key, msg, out);
}

/* rows x r int8 in [-32, 31] (reference.py:74-79): byte b of hash h gives (b & 63) - 32. */
void orc_uniform_matrix(const uint32_t label[8], const uint32_t key[8], uint64_t rows, uint32_t r, int8_t* out) {
  uint64_t nblk = rows * r / 32;
  for (uint64_t b = 0; b < nblk; b++) {
    uint32_t h[8];
    orc_random_hash((uint32_t)b, label, key, 0, h);
    for (int i = 0; i < 32; i++) out[b * 32 + i] = (int8_t)((int)((h[i / 4] >> (8 * (i % 4))) & 63u) - 32);
  }
}

/* k pairs, packed first | second << 16 (reference.py:82-93):
 * first = u & (r-1), second = first ^ (1 + mulhi32(r-1, u)). */
void orc_perm_matrix(const uint32_t label[8], const uint32_t key[8], uint32_t k, uint32_t r, uint32_t* out) {
  for (uint32_t i = 0; i * 8 < k; i++) {
    uint32_t h[8];
    orc_random_hash(i, label, key, 1, h);
    for (int j = 0; j < 8; j++) {
      uint32_t l = i * 8 + j;
      if (l >= k) break;
      uint32_t u = h[j];
      uint32_t first = u & (r - 1);
      uint32_t second = first ^ (1u + (uint32_t)(((uint64_t)(r - 1) * u) >> 32));
      out[l] = first | (second << 16);
    }
  }
}

/* noise_rows semantics (kernels.cu:303-372):
 *   dst[i,l]  = src[i,l] + E[i, Pn.first(l)] - E[i, Pn.second(l)]        (if dst)
 *   proj[i,j] = sum_l src[i,l] ([Pp.first(l)=j] - [Pp.second(l)=j])      (if Pp)
 *   corr[li][i][corr_off + j] = balanced base-128 limb li of proj[i,j]   (if Pp and corr_off >= 0)
 *   corr[li][i][ecopy_off + j] = E[i,j]                                  (if E and ecopy_off >= 0)
 *   *maxabs = max(*maxabs, max |proj|)                                     (if Pp and maxabs)
 * corr rows have stride 2r; limb li starts at li * rows * 2r. */
void orc_noise_rows(const int8_t* src, int rows, int k, int r, const int8_t* E, const uint32_t* Pn, int8_t* dst,
                    const uint32_t* Pp, int8_t* corr, int corr_off, int ecopy_off, int32_t* maxabs, int lmax) {
  int64_t* proj = (int64_t*)calloc((size_t)r, sizeof(int64_t));
  uint64_t limb_stride = (uint64_t)rows * 2 * r;
  int32_t mx = maxabs ? *maxabs : 0;
  for (int i = 0; i < rows; i++) {
    const int8_t* s = src + (uint64_t)i * k;
    if (dst) {
      const int8_t* e = E + (uint64_t)i * r;
      for (int l = 0; l < k; l++) {
        int v = s[l] + e[Pn[l] & 0xFFFF] - e[Pn[l] >> 16];
        dst[(uint64_t)i * k + l] = (int8_t)v;
      }
    }
    if (Pp) {
      memset(proj, 0, sizeof(int64_t) * r);
      for (int l = 0; l < k; l++) {
        proj[Pp[l] & 0xFFFF] += s[l];
        proj[Pp[l] >> 16] -= s[l];
      }
      for (int j = 0; j < r; j++) {
        int64_t v = proj[j];
        int32_t a = (int32_t)(v < 0 ? -v : v);
        if (a > mx) mx = a;
        if (corr && corr_off >= 0) {
          for (int li = 0; li < lmax; li++) {
            int64_t d = ((v + 64) & 127) - 64;
            corr[li * limb_stride + (uint64_t)i * 2 * r + corr_off + j] = (int8_t)d;
            v = (v - d) >> 7;
          }
        }
      }
    }
    if (E && corr && ecopy_off >= 0) {
      for (int li = 0; li < lmax; li++)
        memcpy(corr + li * limb_stride + (uint64_t)i * 2 * r + ecopy_off, E + (uint64_t)i * r, (size_t)r);
    }
  }
  if (maxabs && Pp) *maxabs = mx;
  free(proj);
}

/* Balanced base-128 limbs that always cover |projection| <= 127 k (ops.py:18-24). */
int orc_limbs_for(int k) {
  int64_t bound = 127LL * k, cap = 63;
  int L = 1;
  while (cap < bound) {
    L++;
    cap = cap * 128 + 63;
  }
  return L;
}

/* ------------------------------------------------------------------ jackpot fold */
/* Hash tile (rb, g, cb, t) = rows rb*64 + g + 8i (i<8), cols cb*64 + 8j + 2t + e (j<8, e<2)
 * (pearl_glue.py:14-15).  msgs layout: [(m/64)*8 + g ... ] flattened as
 * msgs[(((rb * 8 + g) * (n/64) + cb) * 4 + t) * 16 + w]  (matches reference.py:138-165 shapes). */
typedef struct {
  const int8_t *Ap, *Bp;
  int m, n, k, r, t0, t1, ncs;
  uint32_t* msgs;
} fold_job;

/* Work item w = (row block rb, column stripe cs): 64 rows x a stripe of 64-column blocks. Items are
 * independent (each hash tile lives in exactly one), so threads split them freely. */
static void* fold_worker(void* arg) {
  fold_job* j = (fold_job*)arg;
  const int n = j->n, k = j->k, r = j->r, nch = k / r, ncb = n / 64, ncs = j->ncs;
  const int cbs = (ncb + ncs - 1) / ncs;  /* 64-column blocks per stripe */
  int32_t* acc = (int32_t*)calloc((size_t)64 * cbs * 64, sizeof(int32_t));
  for (int w = j->t0; w < j->t1; w++) {
    const int rb = w / ncs, cs = w % ncs, cb0 = cs * cbs, cb1 = cb0 + cbs < ncb ? cb0 + cbs : ncb;
    if (cb0 >= cb1) continue;
    const int wc = (cb1 - cb0) * 64, c0 = cb0 * 64;
    memset(acc, 0, sizeof(int32_t) * 64 * wc);
    for (int g = 0; g < 8; g++)
      for (int cb = cb0; cb < cb1; cb++)
        memset(j->msgs + ((((uint64_t)rb * 8 + g) * ncb + cb) * 4) * 16, 0, sizeof(uint32_t) * 4 * 16);
    for (int c = 0; c < nch; c++) {
      for (int i = 0; i < 64; i++) {
        const int8_t* a = j->Ap + (uint64_t)(rb * 64 + i) * k + (uint64_t)c * r;
        int32_t* ar = acc + (uint64_t)i * wc;
        for (int col = 0; col < wc; col++) {
          const int8_t* b = j->Bp + (uint64_t)(c0 + col) * k + (uint64_t)c * r;
          int32_t s = 0;
          for (int l = 0; l < r; l++) s += (int32_t)a[l] * (int32_t)b[l];
          ar[col] = (int32_t)((uint32_t)ar[col] + (uint32_t)s);
        }
      }
      const int slot = c % 16;
      for (int g = 0; g < 8; g++)
        for (int cb = cb0; cb < cb1; cb++)
          for (int t = 0; t < 4; t++) {
            uint32_t x = 0;
            for (int i = 0; i < 8; i++)
              for (int jj = 0; jj < 8; jj++)
                for (int e = 0; e < 2; e++)
                  x ^= (uint32_t)acc[(uint64_t)(g + 8 * i) * wc + (cb - cb0) * 64 + 8 * jj + 2 * t + e];
            uint32_t* wd = j->msgs + ((((uint64_t)rb * 8 + g) * ncb + cb) * 4 + t) * 16 + slot;
            *wd = ((*wd << 13) | (*wd >> 19)) ^ x;
          }
    }
  }
  free(acc);
  return NULL;
}

/* Ap: m x k, Bp: n x k int8 (noised operands), m % 64 == 0, n % 64 == 0, k % r == 0. */
void orc_jackpot_msgs(const int8_t* Ap, const int8_t* Bp, int m, int n, int k, int r, uint32_t* msgs, int nthreads) {
  const int nrb = m / 64, ncb = n / 64;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 64) nthreads = 64;
  /* enough column stripes that every thread has work even for a few row blocks */
  int ncs = (nthreads * 2 + nrb - 1) / nrb;
  if (ncs > ncb) ncs = ncb;
  if (ncs < 1) ncs = 1;
  const int items = nrb * ncs;
  if (nthreads > items) nthreads = items;
  pthread_t th[64];
  fold_job jobs[64];
  for (int t = 0; t < nthreads; t++) {
    jobs[t] = (fold_job){Ap, Bp, m, n, k, r, (int)((int64_t)items * t / nthreads),
                         (int)((int64_t)items * (t + 1) / nthreads), ncs, msgs};
    pthread_create(&th[t], NULL, fold_worker, &jobs[t]);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* Keyed hash of each tile message; winners are tiles with LE-U256(hash) <= target.
 * rec = {row_off, col_off, hash[8]} (kernels.cu:579-595 record format).  Returns the count
 * (records beyond max_recs are counted but not written). */
int orc_winners(const uint32_t* msgs, int m, int n, const uint32_t a_seed[8], const uint32_t target[8], uint32_t* recs,
                int max_recs) {
  int ncb = n / 64, cnt = 0;
  for (int rb = 0; rb < m / 64; rb++)
    for (int g = 0; g < 8; g++)
      for (int cb = 0; cb < ncb; cb++)
        for (int t = 0; t < 4; t++) {
          const uint32_t* w = msgs + ((((uint64_t)rb * 8 + g) * ncb + cb) * 4 + t) * 16;
          uint32_t h[8];
          orc_b3_hash64(a_seed, w, h);
          int le = 1;
          for (int i = 7; i >= 0; i--)
            if (h[i] != target[i]) {
              le = h[i] < target[i];
              break;
            }
          if (le) {
            if (cnt < max_recs) {
              uint32_t* rec = recs + (uint64_t)cnt * 10;
              rec[0] = (uint32_t)(rb * 64 + g);
              rec[1] = (uint32_t)(cb * 64 + 2 * t);
              memcpy(rec + 2, h, 32);
            }
            cnt++;
          }
        }
  return cnt;
}

/* ------------------------------------------------------------------ exact int32 GEMM */
typedef struct {
  const int8_t *A, *B;
  int m, n, k, r0, r1;
  int32_t* C;
} gemm_job;

static void* gemm_worker(void* arg) {
  gemm_job* j = (gemm_job*)arg;
  for (int i = j->r0; i < j->r1; i++) {
    const int8_t* a = j->A + (uint64_t)i * j->k;
    for (int c = 0; c < j->n; c++) {
      const int8_t* b = j->B + (uint64_t)c * j->k;
      int32_t s = 0;
      for (int l = 0; l < j->k; l++) s += (int32_t)a[l] * (int32_t)b[l];
      j->C[(uint64_t)i * j->n + c] = s;
    }
  }
  return NULL;
}

/* C = A B^T, A m x k, B n x k (int8, k contiguous), int32 out (exact for |C| < 2^31). */
void orc_gemm_i32(const int8_t* A, const int8_t* B, int m, int n, int k, int32_t* C, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > m) nthreads = m;
  if (nthreads > 64) nthreads = 64;
  pthread_t th[64];
  gemm_job jobs[64];
  for (int t = 0; t < nthreads; t++) {
    jobs[t] = (gemm_job){A, B, m, n, k, (int)((int64_t)m * t / nthreads), (int)((int64_t)m * (t + 1) / nthreads), C};
    pthread_create(&th[t], NULL, gemm_worker, &jobs[t]);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}
