// noise_gen.cu -- seeded low-rank noise factors.
//
// Restates zk-pow/src/circuit/pearl_noise.rs (get_random_hash :46-58,
// generate_uniform_random_matrix :61-80, generate_permutation_matrix :90-116)
// with the reference GPU operator's output formats (noise_generation_kernel.h):
// one keyed BLAKE3 compression yields 32 random bytes, which become 32 dense
// values (EAL / EBR, (byte & 63) - 32, plus scaled half copies; one
// compression per thread) or 8 index pairs of a sparse factor (EAR / EBL, +1
// at r0, -1 at r1; 16 compressions per block of 128 k-columns, whose threads
// then write the block's R-major (k,r) and K-major (r,k) dense forms with
// coalesced stores).
#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int kThreads = 128;
constexpr int kSparseK = 128;  // k-columns of a sparse factor per block

struct NoiseArgs {
  pb2_noise_gen_params p;
  int64_t units_eal, units_ebr, units_aux;
  int64_t blocks_eal, blocks_ebr, blocks_ear, blocks_ebl;
};

// Seed label words: "A_tensor" / "B_tensor" zero-padded to 32 bytes.
__device__ __forceinline__ void seed_words(bool b_side, uint32_t* w) {
  w[0] = b_side ? 0x65745f42u : 0x65745f41u;  // "B_te" / "A_te"
  w[1] = 0x726f736eu;                          // "nsor"
#pragma unroll
  for (int i = 2; i < 8; ++i) w[i] = 0;
}

__device__ __forceinline__ void load_key(const uint8_t* key, uint32_t* k) {
  const uint4* p = reinterpret_cast<const uint4*>(key);
  uint4 a = p[0], b = p[1];
  k[0] = a.x; k[1] = a.y; k[2] = a.z; k[3] = a.w;
  k[4] = b.x; k[5] = b.y; k[6] = b.z; k[7] = b.w;
}

// 32 random bytes = keyed BLAKE3 of [8 x le32 slots with (index+1) at `slot`,
// 32-byte seed label].
__device__ __forceinline__ void random_block(const uint8_t* key, bool b_side, int slot,
                                             uint64_t index, uint32_t* out) {
  uint32_t m[16], cv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = 0;
  if (slot == 0) m[0] = uint32_t(index + 1); else m[1] = uint32_t(index + 1);
  seed_words(b_side, m + 8);
  load_key(key, cv);
  b3_compress8(cv, m, kB3SingleBlockKeyed, out);
}

__device__ void dense_unit(const pb2_noise_gen_params& p, bool b_side, int64_t u) {
  const int64_t rows = b_side ? p.n : p.m;
  const int64_t total = rows * p.r;
  if (u * 32 >= total) return;
  uint32_t h[8];
  random_block(b_side ? p.key_b : p.key_a, b_side, 0, uint64_t(u), h);
  // value = (byte & 63) - 32, four bytes per word
  uint32_t vals[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t w = h[i] & 0x3F3F3F3Fu;
    // per-byte subtract 32 (no borrow across bytes: each byte >= 0 after mask)
    vals[i] = __vsub4(w, 0x20202020u);
  }
  int8_t* out = b_side ? p.EBR : p.EAL;
  if (out) {
    uint4* dst = reinterpret_cast<uint4*>(out + u * 32);
    dst[0] = make_uint4(vals[0], vals[1], vals[2], vals[3]);
    dst[1] = make_uint4(vals[4], vals[5], vals[6], vals[7]);
  }
  void* out16 = b_side ? p.EBR_fp16 : p.EAL_fp16;
  if (out16) {
    const float scale = b_side ? -4.0f : -1.0f;  // kEBR/kEALScaleFactorDenoise
    __half2 hv[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int8_t b0 = int8_t(vals[i] & 0xFF), b1 = int8_t((vals[i] >> 8) & 0xFF);
      int8_t b2 = int8_t((vals[i] >> 16) & 0xFF), b3 = int8_t(vals[i] >> 24);
      hv[2 * i] = __floats2half2_rn(float(b0) * scale, float(b1) * scale);
      hv[2 * i + 1] = __floats2half2_rn(float(b2) * scale, float(b3) * scale);
    }
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(out16) + u * 32);
    const uint4* src = reinterpret_cast<const uint4*>(hv);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = src[i];
  }
}

// One block per 128 k-columns of a sparse factor: 16 lanes draw the block's
// 16 units (8 index pairs each) into shared memory, then all threads write
// the R-major rows (k, r) and the K-major column block (r, 128) of the block
// as coalesced 16-byte chunks.
__device__ void sparse_block(const pb2_noise_gen_params& p, bool b_side, int64_t kb) {
  __shared__ int16_t s_r0[kSparseK], s_r1[kSparseK];
  const int t = threadIdx.x;
  const int64_t kbase = kb * kSparseK;
  const int nk = int(min(int64_t(kSparseK), p.k - kbase));  // a multiple of 16
  const int r = int(p.r);
  if (t < kSparseK / 8) {
    const int64_t u = kb * (kSparseK / 8) + t;
    if (u * 8 < p.k) {
      uint32_t h[8];
      random_block(b_side ? p.key_b : p.key_a, b_side, 1, uint64_t(u), h);
      const uint32_t mask = uint32_t(r - 1);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t r0 = h[j] & mask;
        s_r0[8 * t + j] = int16_t(r0);
        s_r1[8 * t + j] = int16_t(r0 ^ (1u + __umulhi(uint32_t(r - 1), h[j])));
      }
    }
  }
  __syncthreads();
  int8_t* rmaj = b_side ? p.EBL_R_major : p.EAR_R_major;
  int8_t* kmaj = b_side ? p.EBL_K_major : p.EAR_K_major;
  if (rmaj) {
    // row kk: +1 at r0[kk], -1 at r1[kk] (r0 != r1)
    const int cpr = r / 16;
    for (int idx = t; idx < nk * cpr; idx += kThreads) {
      const int kk = idx / cpr, c = idx % cpr;
      const int r0 = s_r0[kk], r1 = s_r1[kk];
      uint32_t w[4] = {0, 0, 0, 0};
      if (r0 / 16 == c) w[(r0 % 16) / 4] |= 0x01u << (8 * (r0 % 4));
      if (r1 / 16 == c) w[(r1 % 16) / 4] |= 0xFFu << (8 * (r1 % 4));
      *reinterpret_cast<uint4*>(rmaj + (kbase + kk) * r + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  if (kmaj) {
    // row rr, column kk: [r0[kk] == rr] - [r1[kk] == rr]
    const int cpr = nk / 16;
    for (int idx = t; idx < r * cpr; idx += kThreads) {
      const int rr = idx / cpr, c = idx % cpr;
      uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int kk = 16 * c + j;
        const uint32_t b = (s_r0[kk] == rr) ? 0x01u : ((s_r1[kk] == rr) ? 0xFFu : 0u);
        w[j / 4] |= b << (8 * (j % 4));
      }
      *reinterpret_cast<uint4*>(kmaj + int64_t(rr) * p.k + kbase + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Blocks are assigned whole to one part (dense EAL, dense EBR, sparse EAR,
// sparse EBL, aux clearing), so a sparse block can synchronise.
__global__ void __launch_bounds__(kThreads) noise_gen_kernel(const __grid_constant__ NoiseArgs a) {
  // The factors are read by the previous mined GEMM in the stream: write
  // them only once it has completed.
  griddep_wait();
  griddep_launch_dependents();
  int64_t b = blockIdx.x;
  const int t = threadIdx.x;
  if (b < a.blocks_eal) {
    const int64_t u = b * kThreads + t;
    if (u < a.units_eal) dense_unit(a.p, false, u);
    return;
  }
  b -= a.blocks_eal;
  if (b < a.blocks_ebr) {
    const int64_t u = b * kThreads + t;
    if (u < a.units_ebr) dense_unit(a.p, true, u);
    return;
  }
  b -= a.blocks_ebr;
  if (b < a.blocks_ear) { sparse_block(a.p, false, b); return; }
  b -= a.blocks_ear;
  if (b < a.blocks_ebl) { sparse_block(a.p, true, b); return; }
  b -= a.blocks_ebl;
  const int64_t u = b * kThreads + t;
  if (u < a.units_aux) {
    uint4* dst = reinterpret_cast<uint4*>(a.p.aux_buffer) + u * 2;
    int64_t words = a.p.aux_words - u * 8;
    dst[0] = make_uint4(0, 0, 0, 0);
    if (words > 4) dst[1] = make_uint4(0, 0, 0, 0);
  }
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace
}  // namespace pb2

extern "C" int pb2_noise_gen(const pb2_noise_gen_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_noise_gen");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_noise_gen_params& p = *pp;
  const bool want_a = p.EAL || p.EAL_fp16 || p.EAR_R_major || p.EAR_K_major;
  const bool want_b = p.EBR || p.EBR_fp16 || p.EBL_R_major || p.EBL_K_major;
  if (!want_a && !want_b && !p.aux_buffer) return PB2_ERR_INVALID_ARGUMENT;
  if (want_a && !p.key_a) return PB2_ERR_INVALID_ARGUMENT;
  if (want_b && !p.key_b) return PB2_ERR_INVALID_ARGUMENT;
  if (want_a || want_b) {
    if (!(p.r == 32 || p.r == 64 || p.r == 128 || p.r == 256)) return PB2_ERR_UNSUPPORTED_CONFIG;
  }
  const bool sparse = p.EAR_R_major || p.EAR_K_major || p.EBL_R_major || p.EBL_K_major;
  if (sparse && (p.k <= 0 || p.k % 16 != 0)) return PB2_ERR_INVALID_ARGUMENT;
  if ((p.EAL || p.EAL_fp16) && p.m <= 0) return PB2_ERR_INVALID_ARGUMENT;
  if ((p.EBR || p.EBR_fp16) && p.n <= 0) return PB2_ERR_INVALID_ARGUMENT;
  if (p.aux_buffer && p.aux_words % 4 != 0) return PB2_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {p.EAL, p.EAL_fp16, p.EAR_R_major, p.EAR_K_major, p.EBL_R_major,
                        p.EBL_K_major, p.EBR, p.EBR_fp16, p.key_a, p.key_b, p.aux_buffer};
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;

  NoiseArgs a;
  a.p = p;
  a.units_eal = (p.EAL || p.EAL_fp16) ? (p.m * p.r + 31) / 32 : 0;
  a.units_ebr = (p.EBR || p.EBR_fp16) ? (p.n * p.r + 31) / 32 : 0;
  a.units_aux = p.aux_buffer ? (p.aux_words + 7) / 8 : 0;
  a.blocks_eal = (a.units_eal + kThreads - 1) / kThreads;
  a.blocks_ebr = (a.units_ebr + kThreads - 1) / kThreads;
  a.blocks_ear = (p.EAR_R_major || p.EAR_K_major) ? (p.k + kSparseK - 1) / kSparseK : 0;
  a.blocks_ebl = (p.EBL_R_major || p.EBL_K_major) ? (p.k + kSparseK - 1) / kSparseK : 0;
  const int64_t blocks = a.blocks_eal + a.blocks_ebr + a.blocks_ear + a.blocks_ebl +
                         (a.units_aux + kThreads - 1) / kThreads;
  if (blocks == 0) return PB2_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(blocks), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, noise_gen_kernel, a);
  return launch_status();
}
