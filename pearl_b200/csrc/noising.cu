// noising.cu -- operand noising and denoise-factor projection.
//
// Semantics of the reference operators noise_A / noise_B
// (miner/pearl-gemm/csrc/gemm/pearl_gemm_api.cpp:300-500, docstrings in
// src/pearl_gemm/pearl_gemm_interface.py:122-230):
//   XpE  = X + EL . E_rmajor^T         (rank-r update, int8 wrap)
//   proj = Xs . E_kmajor^T             (Xs = X for noise_A, XpE for noise_B)
// computed for arbitrary int8 factor matrices with dp4a on the CUDA cores.
// Both passes stream X once from HBM; the rank-r work is small (r/4 dp4a per
// element).  Integer projections are accumulated with atomic adds (the caller
// zeroes them, as the reference's split-K path requires); half projections are
// written scaled by 2^-14 (AxEBL) or 2^-12 (EARxBpEB).
#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int kThreads = 256;
constexpr int kTileRows = 64;   // rows of X per block
constexpr int kTileK = 128;     // columns of X per block (operand pass)
constexpr int kSlabK = 64;      // k slab of the projection pass
constexpr int kTileR = 128;     // r columns per block (projection pass)

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
  return __dp4a(int(a), int(b), c);
}

// ---------------------------------------------------------------- XpE pass
// smem: EL tile [64][r+4] and E tile [128][r+4] (4-byte pad: conflict-free
// word reads across rows).
__global__ void __launch_bounds__(kThreads) noise_operand_kernel(
    const int8_t* __restrict__ X, const int8_t* __restrict__ EL,
    const int8_t* __restrict__ E_rmajor, int8_t* __restrict__ XpE, int64_t rows, int64_t k,
    int r) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int rs = r + 4;  // padded row stride in bytes
  uint8_t* sEL = smem;
  uint8_t* sE = smem + kTileRows * rs;
  const int64_t row0 = int64_t(blockIdx.y) * kTileRows;
  const int64_t k0 = int64_t(blockIdx.x) * kTileK;
  const int tid = threadIdx.x;
  const int words = r / 4;
  for (int i = tid; i < kTileRows * words; i += kThreads) {
    int rr = i / words, w = i % words;
    uint32_t v = 0;
    if (row0 + rr < rows) v = reinterpret_cast<const uint32_t*>(EL + (row0 + rr) * r)[w];
    *reinterpret_cast<uint32_t*>(sEL + rr * rs + 4 * w) = v;
  }
  for (int i = tid; i < kTileK * words; i += kThreads) {
    int kk = i / words, w = i % words;
    uint32_t v = 0;
    if (k0 + kk < k) v = reinterpret_cast<const uint32_t*>(E_rmajor + (k0 + kk) * r)[w];
    *reinterpret_cast<uint32_t*>(sE + kk * rs + 4 * w) = v;
  }
  __syncthreads();
  const int ty = tid / 16, tx = tid % 16;
  int acc[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[a][b] = 0;
  for (int w = 0; w < words; ++w) {
    uint32_t av[4], bv[8];
#pragma unroll
    for (int a = 0; a < 4; ++a) av[a] = *reinterpret_cast<const uint32_t*>(sEL + (ty * 4 + a) * rs + 4 * w);
#pragma unroll
    for (int b = 0; b < 8; ++b) bv[b] = *reinterpret_cast<const uint32_t*>(sE + (tx + 16 * b) * rs + 4 * w);
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) acc[a][b] = dp4a(av[a], bv[b], acc[a][b]);
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t row = row0 + ty * 4 + a;
    if (row >= rows) continue;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int64_t col = k0 + tx + 16 * b;
      if (col < k) XpE[row * k + col] = int8_t(int(X[row * k + col]) + acc[a][b]);
    }
  }
}

// ---------------------------------------------------------- projection pass
// proj[row][rr] = sum_k Xs[row][k] * E_kmajor[rr][k] over this block's k range.
__global__ void __launch_bounds__(kThreads) noise_project_kernel(
    const int8_t* __restrict__ Xs, const int8_t* __restrict__ E_kmajor, void* __restrict__ proj,
    int64_t rows, int64_t k, int r, int64_t k_per_split, int out_fp16, float scale) {
  __shared__ __align__(16) uint8_t sX[kTileRows][kSlabK + 4];
  __shared__ __align__(16) uint8_t sE[kTileR][kSlabK + 4];
  const int64_t row0 = int64_t(blockIdx.x) * kTileRows;
  const int r0 = blockIdx.y * kTileR;
  const int64_t kb = int64_t(blockIdx.z) * k_per_split;
  const int64_t ke = min(k, kb + k_per_split);
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  int acc[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[a][b] = 0;
  for (int64_t ks = kb; ks < ke; ks += kSlabK) {
    __syncthreads();
    for (int i = tid; i < kTileRows * (kSlabK / 16); i += kThreads) {
      int rr = i / (kSlabK / 16), c = i % (kSlabK / 16);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (row0 + rr < rows && ks + 16 * c < ke)
        v = *reinterpret_cast<const uint4*>(Xs + (row0 + rr) * k + ks + 16 * c);
      uint32_t* d = reinterpret_cast<uint32_t*>(&sX[rr][16 * c]);
      d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
    for (int i = tid; i < kTileR * (kSlabK / 16); i += kThreads) {
      int rr = i / (kSlabK / 16), c = i % (kSlabK / 16);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r0 + rr < r && ks + 16 * c < ke)
        v = *reinterpret_cast<const uint4*>(E_kmajor + int64_t(r0 + rr) * k + ks + 16 * c);
      uint32_t* d = reinterpret_cast<uint32_t*>(&sE[rr][16 * c]);
      d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
    __syncthreads();
#pragma unroll 4
    for (int w = 0; w < kSlabK / 4; ++w) {
      uint32_t av[4], bv[8];
#pragma unroll
      for (int a = 0; a < 4; ++a) av[a] = *reinterpret_cast<const uint32_t*>(&sX[ty * 4 + a][4 * w]);
#pragma unroll
      for (int b = 0; b < 8; ++b) bv[b] = *reinterpret_cast<const uint32_t*>(&sE[tx + 16 * b][4 * w]);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = dp4a(av[a], bv[b], acc[a][b]);
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t row = row0 + ty * 4 + a;
    if (row >= rows) continue;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int rr = r0 + tx + 16 * b;
      if (rr >= r) continue;
      if (out_fp16)
        static_cast<__half*>(proj)[row * r + rr] = __float2half_rn(float(acc[a][b]) * scale);
      else
        atomicAdd(static_cast<int*>(proj) + row * r + rr, acc[a][b]);
    }
  }
}

int run_noising(const pb2_noising_params& p, bool b_side, cudaStream_t stream) {
  if (!p.X || !p.EL || !p.E_rmajor || !p.E_kmajor || !p.XpE || !p.proj)
    return PB2_ERR_INVALID_ARGUMENT;
  if (p.rows <= 0 || p.k <= 0 || p.k % 16 != 0) return PB2_ERR_INVALID_ARGUMENT;
  if (!(p.r == 32 || p.r == 64 || p.r == 128 || p.r == 256)) return PB2_ERR_UNSUPPORTED_CONFIG;
  const void* ptrs[] = {p.X, p.EL, p.E_rmajor, p.E_kmajor, p.XpE, p.proj};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) % 16) return PB2_ERR_INVALID_ARGUMENT;
  if (p.proj_is_fp16 && p.k_blocks_per_split > 0) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  const int r = int(p.r);
  // operand pass
  {
    dim3 grid(unsigned((p.k + kTileK - 1) / kTileK), unsigned((p.rows + kTileRows - 1) / kTileRows));
    size_t smem = size_t(kTileRows + kTileK) * (r + 4);
    if (smem > 48 * 1024) {
      cudaFuncSetAttribute(noise_operand_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(smem));
    }
    noise_operand_kernel<<<grid, kThreads, smem, stream>>>(p.X, p.EL, p.E_rmajor, p.XpE, p.rows,
                                                          p.k, r);
    st = launch_status();
    if (st) return st;
  }
  // projection pass: noise_A projects A, noise_B projects the noised B.
  {
    const int8_t* Xs = b_side ? p.XpE : p.X;
    const int64_t row_blocks = (p.rows + kTileRows - 1) / kTileRows;
    const int r_blocks = (r + kTileR - 1) / kTileR;
    int64_t k_per_split = p.k;
    if (!p.proj_is_fp16) {
      int64_t kbps = p.k_blocks_per_split;
      if (kbps < 0) {
        // enough splits for ~4 blocks per SM
        const int64_t want = 4 * int64_t(sm_count(p.device));
        int64_t splits = (want + row_blocks * r_blocks - 1) / (row_blocks * r_blocks);
        const int64_t kblocks = (p.k + 127) / 128;
        splits = splits < 1 ? 1 : (splits > kblocks ? kblocks : splits);
        kbps = (kblocks + splits - 1) / splits;
      }
      if (kbps > 0) k_per_split = kbps * 128;
    }
    const int64_t splits = (p.k + k_per_split - 1) / k_per_split;
    const dim3 grid = dim3(unsigned(row_blocks), unsigned(r_blocks), unsigned(splits));
    const float scale = b_side ? (1.0f / 4096.0f) : (1.0f / 16384.0f);
    noise_project_kernel<<<grid, kThreads, 0, stream>>>(Xs, p.E_kmajor, p.proj, p.rows, p.k, r,
                                                       k_per_split, p.proj_is_fp16, scale);
    st = launch_status();
  }
  return st;
}

__global__ void denoise_convert_kernel(const int32_t* __restrict__ in, __half* __restrict__ out,
                                       int64_t count, float scale) {
  int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i >= count) return;
  int4 v = *reinterpret_cast<const int4*>(in + i);
  __half2 a = __floats2half2_rn(float(v.x) * scale, float(v.y) * scale);
  __half2 b = __floats2half2_rn(float(v.z) * scale, float(v.w) * scale);
  uint2 o;
  o.x = *reinterpret_cast<uint32_t*>(&a);
  o.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(out + i) = o;
}

}  // namespace

int denoise_convert(const int32_t* in, void* out, int64_t count, float scale, cudaStream_t s) {
  if (count % 4 != 0) return PB2_ERR_INVALID_ARGUMENT;
  const int64_t threads = count / 4;
  denoise_convert_kernel<<<unsigned((threads + 255) / 256), 256, 0, s>>>(
      in, static_cast<__half*>(out), count, scale);
  return launch_status();
}

}  // namespace pb2

extern "C" int pb2_noise_A(const pb2_noising_params* p, void* stream) {
  if (!p) return PB2_ERR_INVALID_ARGUMENT;
  return pb2::run_noising(*p, false, static_cast<cudaStream_t>(stream));
}

extern "C" int pb2_noise_B(const pb2_noising_params* p, void* stream) {
  if (!p) return PB2_ERR_INVALID_ARGUMENT;
  return pb2::run_noising(*p, true, static_cast<cudaStream_t>(stream));
}

extern "C" int pb2_denoise_converter(const pb2_denoise_converter_params* pp, void* stream) {
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const auto& p = *pp;
  const bool do_b = p.EARxBpEB_in && p.EARxBpEB_out;
  const bool do_a = p.AxEBL_in && p.AxEBL_out;
  if (!do_a && !do_b) return PB2_ERR_INVALID_ARGUMENT;
  if (!(p.r == 64 || p.r == 128 || p.r == 32 || p.r == 256)) return PB2_ERR_UNSUPPORTED_CONFIG;
  int st = set_device(p.device);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (do_a && (st = denoise_convert(p.AxEBL_in, p.AxEBL_out, p.m * p.r, 1.0f / 16384.0f, s)))
    return st;
  if (do_b && (st = denoise_convert(p.EARxBpEB_in, p.EARxBpEB_out, p.n * p.r, 1.0f / 4096.0f, s)))
    return st;
  return PB2_OK;
}
