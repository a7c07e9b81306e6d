/*
 * pearl_oracle.c -- CPU restatement of Pearl's mining arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the
 * B200 kernels in pearl_b200/csrc and the timed CPU baseline in bench.py.
 * Nothing in the product path links, loads or calls it.
 *
 * Each function cites the reference code it restates (paths relative to the
 * pearl-research-labs/pearl repository).  BLAKE3 itself lives in the `blake3`
 * Rust crate (1.8.x, not vendored in the reference); it is restated here from
 * the published BLAKE3 specification and pinned against the Python `blake3`
 * package by the tests.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define PO_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* BLAKE3 (published specification: 7-round ChaCha-like compression, 1 KiB   */
/* chunks, binary tree of parent nodes).                                     */
/* ------------------------------------------------------------------------- */

enum {
  B3_CHUNK_START = 1,
  B3_CHUNK_END = 2,
  B3_PARENT = 4,
  B3_ROOT = 8,
  B3_KEYED_HASH = 16,
};

static const uint32_t B3_IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u,
                                  0xA54FF53Au, 0x510E527Fu, 0x9B05688Cu,
                                  0x1F83D9ABu, 0x5BE0CD19u};

static const uint8_t B3_PERM[16] = {2, 6,  3,  10, 7, 0,  4,  13,
                                    1, 11, 12, 5,  9, 14, 15, 8};

static inline uint32_t rotr32(uint32_t x, int n) {
  return (x >> n) | (x << (32 - n));
}

static inline void b3_g(uint32_t* v, int a, int b, int c, int d, uint32_t mx,
                        uint32_t my) {
  v[a] = v[a] + v[b] + mx;
  v[d] = rotr32(v[d] ^ v[a], 16);
  v[c] = v[c] + v[d];
  v[b] = rotr32(v[b] ^ v[c], 12);
  v[a] = v[a] + v[b] + my;
  v[d] = rotr32(v[d] ^ v[a], 8);
  v[c] = v[c] + v[d];
  v[b] = rotr32(v[b] ^ v[c], 7);
}

/* Full 16-word compression output. */
PO_EXPORT void po_blake3_compress(const uint32_t cv[8], const uint32_t block[16],
                                  uint64_t counter, uint32_t block_len,
                                  uint32_t flags, uint32_t out[16]) {
  uint32_t v[16];
  uint32_t m[16];
  memcpy(m, block, sizeof(m));
  for (int i = 0; i < 8; ++i) v[i] = cv[i];
  v[8] = B3_IV[0];
  v[9] = B3_IV[1];
  v[10] = B3_IV[2];
  v[11] = B3_IV[3];
  v[12] = (uint32_t)counter;
  v[13] = (uint32_t)(counter >> 32);
  v[14] = block_len;
  v[15] = flags;
  for (int r = 0; r < 7; ++r) {
    b3_g(v, 0, 4, 8, 12, m[0], m[1]);
    b3_g(v, 1, 5, 9, 13, m[2], m[3]);
    b3_g(v, 2, 6, 10, 14, m[4], m[5]);
    b3_g(v, 3, 7, 11, 15, m[6], m[7]);
    b3_g(v, 0, 5, 10, 15, m[8], m[9]);
    b3_g(v, 1, 6, 11, 12, m[10], m[11]);
    b3_g(v, 2, 7, 8, 13, m[12], m[13]);
    b3_g(v, 3, 4, 9, 14, m[14], m[15]);
    if (r < 6) {
      uint32_t t[16];
      for (int i = 0; i < 16; ++i) t[i] = m[B3_PERM[i]];
      memcpy(m, t, sizeof(m));
    }
  }
  for (int i = 0; i < 8; ++i) {
    out[i] = v[i] ^ v[i + 8];
    out[i + 8] = v[i + 8] ^ cv[i];
  }
}

static inline uint32_t load_le32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
         ((uint32_t)p[3] << 24);
}

static inline void store_le32(uint8_t* p, uint32_t x) {
  p[0] = (uint8_t)x;
  p[1] = (uint8_t)(x >> 8);
  p[2] = (uint8_t)(x >> 16);
  p[3] = (uint8_t)(x >> 24);
}

/* Chaining value of one chunk (<= 1024 bytes).  `root` adds ROOT to the last
 * block (only when the whole input is this single chunk). */
static void b3_chunk_cv(const uint32_t key[8], uint32_t base_flags,
                        const uint8_t* data, size_t len, uint64_t chunk_index,
                        int root, uint32_t cv_out[8]) {
  uint32_t cv[8];
  memcpy(cv, key, sizeof(cv));
  size_t nblocks = len == 0 ? 1 : (len + 63) / 64;
  for (size_t b = 0; b < nblocks; ++b) {
    uint8_t buf[64];
    memset(buf, 0, sizeof(buf));
    size_t off = b * 64;
    size_t blen = len - off < 64 ? len - off : 64;
    if (len == 0) blen = 0;
    if (blen) memcpy(buf, data + off, blen);
    uint32_t m[16];
    for (int i = 0; i < 16; ++i) m[i] = load_le32(buf + 4 * i);
    uint32_t flags = base_flags;
    if (b == 0) flags |= B3_CHUNK_START;
    if (b == nblocks - 1) {
      flags |= B3_CHUNK_END;
      if (root) flags |= B3_ROOT;
    }
    uint32_t out[16];
    po_blake3_compress(cv, m, chunk_index, (uint32_t)blen, flags, out);
    memcpy(cv, out, sizeof(cv));
  }
  memcpy(cv_out, cv, sizeof(cv));
}

static void b3_parent_cv(const uint32_t key[8], uint32_t base_flags,
                         const uint32_t left[8], const uint32_t right[8],
                         int root, uint32_t cv_out[8]) {
  uint32_t m[16];
  memcpy(m, left, 32);
  memcpy(m + 8, right, 32);
  uint32_t out[16];
  po_blake3_compress(key, m, 0, 64, base_flags | B3_PARENT | (root ? B3_ROOT : 0),
                     out);
  memcpy(cv_out, out, 32);
}

/* CV of the subtree over chunks [first, first+n).  The left subtree holds the
 * largest power of two number of chunks that leaves >= 1 chunk on the right. */
static void b3_subtree(const uint32_t key[8], uint32_t base_flags,
                       const uint8_t* data, size_t len, uint64_t first,
                       uint64_t n, int root, uint32_t cv_out[8]) {
  if (n == 1) {
    size_t off = (size_t)first * 1024;
    size_t clen = len - off < 1024 ? len - off : 1024;
    b3_chunk_cv(key, base_flags, data + off, clen, first, root, cv_out);
    return;
  }
  uint64_t left_n = 1;
  while (left_n * 2 < n) left_n *= 2;
  uint32_t l[8], r[8];
  b3_subtree(key, base_flags, data, len, first, left_n, 0, l);
  b3_subtree(key, base_flags, data, len, first + left_n, n - left_n, 0, r);
  b3_parent_cv(key, base_flags, l, r, root, cv_out);
}

/* blake3(data) or blake3_keyed(key, data): 32-byte digest.
 * Restates pearl-blake3/src/hasher.rs:183-188 (blake3_digest). */
PO_EXPORT void po_blake3(const uint8_t* data, size_t len, const uint8_t* key32,
                         uint8_t out32[32]) {
  uint32_t key[8];
  uint32_t flags = 0;
  if (key32) {
    for (int i = 0; i < 8; ++i) key[i] = load_le32(key32 + 4 * i);
    flags = B3_KEYED_HASH;
  } else {
    memcpy(key, B3_IV, sizeof(key));
  }
  uint64_t nchunks = len == 0 ? 1 : (len + 1023) / 1024;
  uint32_t cv[8];
  b3_subtree(key, flags, data, len, 0, nchunks, 1, cv);
  for (int i = 0; i < 8; ++i) store_le32(out32 + 4 * i, cv[i]);
}

/* ------------------------------------------------------------------------- */
/* Noise generation: zk-pow/src/circuit/pearl_noise.rs                       */
/* ------------------------------------------------------------------------- */

/* Seed labels "A_tensor"/"B_tensor" zero-padded to 32 bytes
 * (pearl_noise.rs:29-30; noise_generation_kernel.h:717-718). */
static void seed_label(int which_b, uint8_t out[32]) {
  memset(out, 0, 32);
  memcpy(out, which_b ? "B_tensor" : "A_tensor", 8);
}

/* get_random_hash (pearl_noise.rs:46-58): message = 8 little-endian i32 slots
 * with (1 + index) at `prepend_slot`, then the 32-byte seed; keyed by `key`. */
static void random_hash(uint64_t index, const uint8_t seed[32],
                        const uint8_t key[32], int prepend_slot,
                        uint8_t out[32]) {
  uint8_t msg[64];
  memset(msg, 0, sizeof(msg));
  store_le32(msg + 4 * prepend_slot, (uint32_t)(int32_t)(1 + index));
  memcpy(msg + 32, seed, 32);
  po_blake3(msg, 64, key, out);
}

/* Dense factor (EAL rows x R, or EBR rows x R), row-major.
 * generate_uniform_random_matrix (pearl_noise.rs:61-80):
 * value = (byte & 63) - 32, bytes taken from consecutive 32-byte digests of the
 * flattened matrix. */
PO_EXPORT void po_noise_dense(const uint8_t key[32], int which_b, int64_t rows,
                              int64_t r, int8_t* out) {
  uint8_t seed[32];
  seed_label(which_b, seed);
  int64_t total = rows * r;
  int64_t nblocks = (total + 31) / 32;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nblocks; ++b) {
    uint8_t h[32];
    random_hash((uint64_t)b, seed, key, 0, h);
    for (int j = 0; j < 32; ++j) {
      int64_t idx = b * 32 + j;
      if (idx < total) out[idx] = (int8_t)((h[j] & 63) - 32);
    }
  }
}

/* Sparse factor as index pairs (k x 2): row k of EAR^T (or EBL) has +1 at
 * pairs[k][0] and -1 at pairs[k][1].  generate_permutation_matrix
 * (pearl_noise.rs:90-116): per little-endian u32 `u` of the digest,
 * r0 = u & (R-1), r1 = r0 ^ (1 + mulhi(R-1, u)). */
PO_EXPORT void po_noise_pairs(const uint8_t key[32], int which_b, int64_t k,
                              int64_t r, uint8_t* pairs) {
  uint8_t seed[32];
  seed_label(which_b, seed);
  int64_t nblocks = (k + 7) / 8;
  uint32_t mask = (uint32_t)(r - 1);
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nblocks; ++b) {
    uint8_t h[32];
    random_hash((uint64_t)b, seed, key, 1, h);
    for (int j = 0; j < 8; ++j) {
      int64_t kk = b * 8 + j;
      if (kk >= k) break;
      uint32_t u = load_le32(h + 4 * j);
      uint32_t r0 = u & mask;
      uint32_t hi = (uint32_t)(((uint64_t)(uint32_t)(r - 1) * u) >> 32);
      uint32_t r1 = r0 ^ (1u + hi);
      pairs[2 * kk] = (uint8_t)r0;
      pairs[2 * kk + 1] = (uint8_t)r1;
    }
  }
}

/* ------------------------------------------------------------------------- */
/* Noising: the dense forms of the reference's noise_A / noise_B operators.  */
/*   ApEA   = A + EAL . EAR_R_major^T     (m x k, int8 wrap like the kernel)  */
/*   AxEBL  = A . EBL_R_major             (m x r, int32)                      */
/*   BpEB   = B + EBR . EBL_R_major^T     (n x k)                             */
/*   EARxBpEB = BpEB . EAR_R_major        (n x r, int32)                      */
/* with the sparse factors given as index pairs (pearl_noise.rs:34-43 style). */
/* Reference semantics: pearl_gemm_interface.py noise_A/noise_B docstrings,  */
/* tests/test_pearl_gemm.py:164-213.                                         */
/* ------------------------------------------------------------------------- */

PO_EXPORT void po_noise_operand(const int8_t* x, const int8_t* el, int64_t rows,
                                int64_t k, int64_t r, const uint8_t* pairs,
                                int8_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    const int8_t* e = el + i * r;
    for (int64_t kk = 0; kk < k; ++kk) {
      int32_t v = x[i * k + kk] + e[pairs[2 * kk]] - e[pairs[2 * kk + 1]];
      out[i * k + kk] = (int8_t)v;
    }
  }
}

/* out[i][r] = sum_k x[i][k] * S[k][r] where S is the +1/-1 pair matrix. */
PO_EXPORT void po_times_pairs(const int8_t* x, int64_t rows, int64_t k,
                              int64_t r, const uint8_t* pairs, int32_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < rows; ++i) {
    int32_t* o = out + i * r;
    for (int64_t j = 0; j < r; ++j) o[j] = 0;
    for (int64_t kk = 0; kk < k; ++kk) {
      int32_t v = x[i * k + kk];
      o[pairs[2 * kk]] += v;
      o[pairs[2 * kk + 1]] -= v;
    }
  }
}

/* ------------------------------------------------------------------------- */
/* Jackpot transcripts.                                                      */
/* zk-pow/src/ffi/mine.rs:86-107 and circuit/chip/jackpot/helper.rs:9-35:    */
/*   for ll in (R..=K).step_by(R):                                           */
/*     acc[u][v] += sum_{l in [ll-R, ll)} a'[row_u][l] * b'[col_v][l]        */
/*     x = XOR of all acc[u][v] (as u32)                                     */
/*     tid = (ll/R - 1) % 16;  T[tid] = rotl(T[tid], 13) ^ x                 */
/* Hash tiles come from threads_partition (mine.rs:485-497) with the miner's */
/* patterns: rows {0,8} (period 16), cols {0,1,8,9,...,248,249} (period 256) */
/* (miner-base settings.py:20-26).  Tile (t_row, t_col) covers rows          */
/* {o_r, o_r+8} and cols {o_c + 8j, o_c + 8j + 1 : j < 32} with              */
/* o_r = 16*(t_row/8) + t_row%8 and o_c = 256*(t_col/4) + 2*(t_col%4).       */
/* ------------------------------------------------------------------------- */

static inline uint32_t rotl32(uint32_t x, int n) {
  return (x << n) | (x >> (32 - n));
}

static inline uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* One hash tile given explicit row and column index lists (h rows, w cols).
 * acc_f32 != 0: the words folded are the float32 bit patterns of the
 * accumulators (this build's FP8 mined GEMM accumulates in f32; exact, and
 * so order-independent, only while every partial sum stays below 2^24). */
static void jackpot_tile_mode(const int8_t* ap, const int8_t* bp, int64_t k,
                              int64_t r, const int64_t* rows, int h,
                              const int64_t* cols, int w, int acc_f32,
                              uint32_t out[16]) {
  int32_t acc[2 * 64];
  int32_t* accp = acc;
  int32_t* heap = NULL;
  if (h * w > 128) {
    heap = (int32_t*)calloc((size_t)h * w, sizeof(int32_t));
    accp = heap;
  } else {
    memset(acc, 0, sizeof(acc));
  }
  uint32_t t[16];
  memset(t, 0, sizeof(t));
  for (int64_t ll = r; ll <= k; ll += r) {
    uint32_t x = 0;
    for (int u = 0; u < h; ++u) {
      const int8_t* arow = ap + rows[u] * k;
      for (int v = 0; v < w; ++v) {
        const int8_t* brow = bp + cols[v] * k;
        int32_t s = 0;
        for (int64_t l = ll - r; l < ll; ++l) s += (int32_t)arow[l] * (int32_t)brow[l];
        accp[u * w + v] += s;
        x ^= acc_f32 ? f32_bits((float)accp[u * w + v]) : (uint32_t)accp[u * w + v];
      }
    }
    int tid = (int)((ll / r - 1) % 16);
    t[tid] = rotl32(t[tid], 13) ^ x;
  }
  memcpy(out, t, sizeof(t));
  free(heap);
}

PO_EXPORT void po_jackpot_tile(const int8_t* ap, const int8_t* bp, int64_t k,
                               int64_t r, const int64_t* rows, int h,
                               const int64_t* cols, int w, uint32_t out[16]) {
  jackpot_tile_mode(ap, bp, k, r, rows, h, cols, w, 0, out);
}

/* Jackpot hash (zk-pow/src/api/proof_utils.rs:1511-1514): keyed BLAKE3 of
 * the 64-byte little-endian transcript, key = A's noise seed. */
PO_EXPORT void po_jackpot_hash(const uint32_t t[16], const uint8_t key[32],
                               uint32_t out[8]) {
  uint8_t msg[64];
  for (int i = 0; i < 16; ++i) store_le32(msg + 4 * i, t[i]);
  uint8_t h[32];
  po_blake3(msg, 64, key, h);
  for (int i = 0; i < 8; ++i) out[i] = load_le32(h + 4 * i);
}

/* U256 (8 little-endian words) compare: hash <= target
 * (mine.rs:109, U256::from_little_endian; pow_utils.hpp:222-231). */
PO_EXPORT int po_u256_le(const uint32_t a[8], const uint32_t b[8]) {
  for (int i = 7; i >= 0; --i) {
    if (a[i] < b[i]) return 1;
    if (a[i] > b[i]) return 0;
  }
  return 1;
}

/* All protocol hash tiles of an m x n GEMM (m % 16 == 0, n % 256 == 0, as
 * threads_partition requires).  Tile index = t_row * (n/64) + t_col where
 * t_row in [0, m/2) and t_col in [0, n/64).  Writes transcripts (16 words),
 * digests (8 words) and hit flags for tiles [tile_begin, tile_end). */
static void mine_tiles_mode(const int8_t* ap, const int8_t* bp, int64_t n,
                            int64_t k, int64_t r, const uint8_t key[32],
                            const uint32_t target[8], int64_t tile_begin,
                            int64_t tile_end, int acc_f32, uint32_t* transcripts,
                            uint32_t* digests, uint8_t* hits) {
  int64_t tcols = n / 64;
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t t = tile_begin; t < tile_end; ++t) {
    int64_t trow = t / tcols, tcol = t % tcols;
    int64_t orow = 16 * (trow / 8) + trow % 8;
    int64_t ocol = 256 * (tcol / 4) + 2 * (tcol % 4);
    int64_t rows[2] = {orow, orow + 8};
    int64_t cols[64];
    for (int j = 0; j < 32; ++j) {
      cols[2 * j] = ocol + 8 * j;
      cols[2 * j + 1] = ocol + 8 * j + 1;
    }
    uint32_t tr[16], dg[8];
    jackpot_tile_mode(ap, bp, k, r, rows, 2, cols, 64, acc_f32, tr);
    po_jackpot_hash(tr, key, dg);
    int64_t slot = t - tile_begin;
    if (transcripts) memcpy(transcripts + 16 * slot, tr, sizeof(tr));
    if (digests) memcpy(digests + 8 * slot, dg, sizeof(dg));
    if (hits) hits[slot] = (uint8_t)po_u256_le(dg, target);
  }
}

PO_EXPORT void po_mine_tiles(const int8_t* ap, const int8_t* bp, int64_t m,
                             int64_t n, int64_t k, int64_t r,
                             const uint8_t key[32], const uint32_t target[8],
                             int64_t tile_begin, int64_t tile_end,
                             uint32_t* transcripts, uint32_t* digests,
                             uint8_t* hits) {
  (void)m;
  mine_tiles_mode(ap, bp, n, k, r, key, target, tile_begin, tile_end, 0, transcripts, digests, hits);
}

/* po_mine_tiles over the float32 bit patterns of the accumulators (see
 * jackpot_tile_mode): the operands are the integer values of FP8 elements. */
PO_EXPORT void po_mine_tiles_f32(const int8_t* ap, const int8_t* bp, int64_t m,
                                 int64_t n, int64_t k, int64_t r,
                                 const uint8_t key[32], const uint32_t target[8],
                                 int64_t tile_begin, int64_t tile_end,
                                 uint32_t* transcripts, uint32_t* digests,
                                 uint8_t* hits) {
  (void)m;
  mine_tiles_mode(ap, bp, n, k, r, key, target, tile_begin, tile_end, 1, transcripts, digests, hits);
}

/* ------------------------------------------------------------------------- */
/* Commitment / seed chain.                                                  */
/* zk-pow/src/ffi/mine.rs:442-479 (compute_commitment_hash_with_offsets),    */
/* api/proof_utils.rs:361-372 (commitment_hash), api/seed.rs:20-58           */
/* (legacy vs salted roots), proof_utils.rs:34-45 (MoE routing fold).        */
/* ------------------------------------------------------------------------- */

/* blake3("pearl/cert-v3/noise-seed/A") and ".../B" (api/seed.rs:31-39);
 * derived here at run time instead of hard-coding the constants. */
static void seed_salt(int which_b, uint8_t out[32]) {
  const char* s = which_b ? "pearl/cert-v3/noise-seed/B" : "pearl/cert-v3/noise-seed/A";
  po_blake3((const uint8_t*)s, strlen(s), NULL, out);
}

/* bind_root (seed.rs:41-58): blake3(root || le32(dim) || 28 zero bytes,
 * key = salt). */
static void bind_root(const uint8_t root[32], uint32_t dim, int which_b,
                      uint8_t out[32]) {
  uint8_t salt[32];
  seed_salt(which_b, salt);
  uint8_t msg[64];
  memset(msg, 0, sizeof(msg));
  memcpy(msg, root, 32);
  store_le32(msg + 32, dim);
  po_blake3(msg, 64, salt, out);
}

/* compute_hash_activations (proof_utils.rs:34-45). */
PO_EXPORT void po_hash_activations(const uint8_t hash_a[32],
                                   const uint8_t hash_routing_data[32],
                                   const uint32_t* offsets, int64_t noffsets,
                                   const uint8_t job_key[32], uint8_t out[32]) {
  size_t raw = (size_t)noffsets * 4;
  size_t padded = raw == 0 ? 0 : ((raw + 1023) / 1024) * 1024;
  uint8_t* buf = (uint8_t*)calloc(padded ? padded : 1, 1);
  for (int64_t i = 0; i < noffsets; ++i) store_le32(buf + 4 * i, offsets[i]);
  uint8_t hash_offsets[32], hash_routing[32], cat[64];
  po_blake3(buf, padded, job_key, hash_offsets);
  free(buf);
  memcpy(cat, hash_routing_data, 32);
  memcpy(cat + 32, hash_offsets, 32);
  po_blake3(cat, 64, NULL, hash_routing);
  memcpy(cat, hash_a, 32);
  memcpy(cat + 32, hash_routing, 32);
  po_blake3(cat, 64, NULL, out);
}

/* (b_noise_seed, a_noise_seed) from the two Merkle roots.
 * salted != 0 selects SeedDerivation::Salted with dims (m, n).
 * hash_activations, when non-NULL, replaces hash_a after salting (MoE). */
PO_EXPORT void po_commitment(const uint8_t job_key[32], const uint8_t hash_a[32],
                             const uint8_t hash_b[32], int salted, uint32_t m,
                             uint32_t n, const uint8_t* routing_root,
                             const uint32_t* offsets, int64_t noffsets,
                             uint8_t b_seed[32], uint8_t a_seed[32]) {
  uint8_t ha[32], hb[32], act[32], cat[64];
  if (salted) {
    bind_root(hash_a, m, 0, ha);
    bind_root(hash_b, n, 1, hb);
  } else {
    memcpy(ha, hash_a, 32);
    memcpy(hb, hash_b, 32);
  }
  if (routing_root) {
    po_hash_activations(ha, routing_root, offsets, noffsets, job_key, act);
  } else {
    memcpy(act, ha, 32);
  }
  memcpy(cat, job_key, 32);
  memcpy(cat + 32, hb, 32);
  po_blake3(cat, 64, NULL, b_seed);
  memcpy(cat, b_seed, 32);
  memcpy(cat + 32, act, 32);
  po_blake3(cat, 64, NULL, a_seed);
}

/* Tensor hash = keyed BLAKE3 of the byte tensor zero-padded to a whole number
 * of 1 KiB chunks (pearl-blake3/src/merkle.rs:23-27 pad_to_chunk_boundary;
 * mine.rs:448-452). */
PO_EXPORT void po_tensor_hash(const uint8_t* data, int64_t len,
                              const uint8_t key[32], uint8_t out[32]) {
  int64_t padded = len == 0 ? 0 : ((len + 1023) / 1024) * 1024;
  if (padded == len) {
    po_blake3(data, (size_t)len, key, out);
    return;
  }
  uint8_t* buf = (uint8_t*)calloc((size_t)padded, 1);
  memcpy(buf, data, (size_t)len);
  po_blake3(buf, (size_t)padded, key, out);
  free(buf);
}

/* ------------------------------------------------------------------------- */
/* Merkle tree of a zero-padded tensor: pearl-blake3/src/merkle.rs:43-81      */
/* ------------------------------------------------------------------------- */

static void load_key(const uint8_t key32[32], uint32_t key[8]) {
  for (int i = 0; i < 8; ++i) key[i] = load_le32(key32 + 4 * i);
}

/* Number of nodes over all layers for `len` bytes padded to whole chunks:
 * layer 0 holds one CV per chunk; while a layer has more than two nodes the
 * next one has ceil(n / 2); a two-node layer is followed by the root. */
PO_EXPORT int64_t po_merkle_nodes(int64_t len) {
  int64_t n = (len + 1023) / 1024;
  if (n <= 1) return n;
  int64_t total = n;
  while (n > 2) {
    n = (n + 1) / 2;
    total += n;
  }
  return total + 1;
}

/* CV of 1 KiB chunk `index` (a leaf, never the root). */
PO_EXPORT void po_chunk_cv(const uint8_t key32[32], const uint8_t chunk[1024], uint64_t index,
                           uint8_t out[32]) {
  uint32_t key[8], cv[8];
  load_key(key32, key);
  b3_chunk_cv(key, B3_KEYED_HASH, chunk, 1024, index, 0, cv);
  for (int i = 0; i < 8; ++i) store_le32(out + 4 * i, cv[i]);
}

/* Parent CV of two child CVs; `root` adds the ROOT flag (hasher.rs root_cv). */
PO_EXPORT void po_parent_cv(const uint8_t key32[32], const uint8_t left[32], const uint8_t right[32],
                            int root, uint8_t out[32]) {
  uint32_t key[8], l[8], r[8], cv[8];
  load_key(key32, key);
  for (int i = 0; i < 8; ++i) {
    l[i] = load_le32(left + 4 * i);
    r[i] = load_le32(right + 4 * i);
  }
  b3_parent_cv(key, B3_KEYED_HASH, l, r, root, cv);
  for (int i = 0; i < 8; ++i) store_le32(out + 4 * i, cv[i]);
}

/* All layers, leaves first, 32 bytes per node (po_merkle_nodes(len) nodes).
 * One chunk: the single node is the keyed hash of the padded chunk. */
PO_EXPORT void po_merkle_layers(const uint8_t* data, int64_t len, const uint8_t key32[32],
                                uint8_t* nodes) {
  int64_t n = (len + 1023) / 1024;
  if (n == 0) return;
  uint32_t key[8];
  load_key(key32, key);
  uint8_t chunk[1024];
  for (int64_t c = 0; c < n; ++c) {
    int64_t off = c * 1024, take = len - off < 1024 ? len - off : 1024;
    memset(chunk, 0, sizeof(chunk));
    memcpy(chunk, data + off, (size_t)take);
    uint32_t cv[8];
    b3_chunk_cv(key, B3_KEYED_HASH, chunk, 1024, (uint64_t)c, n == 1, cv);
    for (int i = 0; i < 8; ++i) store_le32(nodes + 32 * c + 4 * i, cv[i]);
  }
  uint8_t* prev = nodes;
  int64_t cnt = n;
  while (cnt > 1) {
    uint8_t* next = prev + 32 * cnt;
    const int root = cnt == 2;
    int64_t pairs = cnt / 2;
    for (int64_t i = 0; i < pairs; ++i)
      po_parent_cv(key32, prev + 64 * i, prev + 64 * i + 32, root, next + 32 * i);
    if (cnt & 1) memcpy(next + 32 * pairs, prev + 32 * (cnt - 1), 32);
    prev = next;
    cnt = pairs + (cnt & 1);
  }
}

PO_EXPORT int po_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

PO_EXPORT void po_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
