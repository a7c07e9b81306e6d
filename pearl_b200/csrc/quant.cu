// quant.cu -- per-token symmetric quantization of the activations that feed
// a mined GEMM: the caller step quant_7bit / quant_8bit of
// miner/vllm-miner/src/vllm_miner/quantization_operators.py:72-100, which
// runs pearl_gemm.quantization.quantize (hadamard.py:530-611).
//
// Per row: x (bf16 / fp16) -> optional block-diagonal Walsh-Hadamard
// transform of width k (Sylvester order, scaled by 1/sqrt(k), first element
// of every block negated: hadamard.py:476-517) -> times the smooth scale ->
// amax; scale = amax * fl(1 / max_val), q = rint(x * inv) clamped to
// [-max_val, max_val] with inv = max_val * rcp.approx.ftz(amax + 1e-30)
// (hadamard.py:443-466): the approximate reciprocal of the reference's
// kernel, so every rounding step, ties included, lands where it does there.
//
// One 256-thread CTA per row, eight elements per thread and 16-byte loads:
// a k-block is k/8 consecutive threads of one warp, so the cross-element
// butterflies are register and shuffle work.  Two passes over the row (amax,
// then quantize); the second pass re-reads the row from L1/L2.  HBM-bound:
// 2 bytes read and 1 written per element.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int kQuantThreads = 256;

struct QuantArgs {
  const void* x;
  const float* smooth;
  int smooth_per_row;
  int8_t* xq;
  float* scales;
  int m, n;
  int block;   // Hadamard width, 0 = none
  float norm;  // 1/sqrt(block), correctly rounded (the reference's constant)
  float max_val;
  float inv_max_val;  // fl(1 / max_val), the reference's compile-time constant
};

// rcp.approx.ftz.f32: the reciprocal the reference's quantizer takes
// (cute.arch.rcp_approx, hadamard.py:446).
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// inv_scale of a row (hadamard.py:443-446).
__device__ __forceinline__ float inv_scale(const QuantArgs& a, float amax) {
  return a.max_val * rcp_approx_ftz(amax + 1e-30f);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// The raw 16 bytes of vector `vec` (8 elements) of `row` (zero when invalid).
template <typename T>
__device__ __forceinline__ uint4 load_raw(const QuantArgs& a, int row, int vec, bool valid) {
  if (!valid) return make_uint4(0u, 0u, 0u, 0u);
  return *reinterpret_cast<const uint4*>(static_cast<const T*>(a.x) + int64_t(row) * a.n + 8 * vec);
}

// Vector `vec` of `row` from its raw bytes: the Hadamard transform of width
// a.block and the smooth scale.  Every lane of the warp must call it with the
// same `iter` (the butterflies shuffle across lanes).
template <typename T>
__device__ __forceinline__ void vec_from_raw(const QuantArgs& a, int row, int vec, bool valid, uint4 raw,
                                             float* v) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = valid ? to_f32<T>(e[i]) : 0.f;
  if (a.block > 0) {
#pragma unroll
    for (int s = 1; s < 8; s <<= 1) {  // butterflies inside the 8-element vector
      float w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = (i & s) ? v[i ^ s] - v[i] : v[i] + v[i ^ s];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = w[i];
    }
    const int lane = threadIdx.x & 31;
    for (int s = 1; 8 * s < a.block; s <<= 1) {  // butterflies across the block's lanes
      const bool upper = lane & s;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float other = __shfl_xor_sync(0xffffffffu, v[i], s);
        v[i] = upper ? other - v[i] : v[i] + other;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] *= a.norm;
    if (vec % (a.block / 8) == 0) v[0] = -v[0];  // first element of the block
  }
  if (a.smooth && valid) {
    const float* sp = a.smooth + (a.smooth_per_row ? int64_t(row) * a.n : 0) + 8 * vec;
    const float4 s0 = *reinterpret_cast<const float4*>(sp);
    const float4 s1 = *reinterpret_cast<const float4*>(sp + 4);
    v[0] *= s0.x; v[1] *= s0.y; v[2] *= s0.z; v[3] *= s0.w;
    v[4] *= s1.x; v[5] *= s1.y; v[6] *= s1.z; v[7] *= s1.w;
  }
}

template <typename T>
__device__ __forceinline__ void load_vec(const QuantArgs& a, int row, int vec, bool valid, float* v) {
  vec_from_raw<T>(a, row, vec, valid, load_raw<T>(a, row, vec, valid), v);
}

template <typename T>
__global__ void __launch_bounds__(kQuantThreads) quant_rows_kernel(const QuantArgs a) {
  __shared__ float warp_max[kQuantThreads / 32];
  griddep_wait();  // launched early behind the previous kernel (programmatic dependent launch)
  griddep_launch_dependents();
  const int row = blockIdx.x;
  const int nvec = a.n / 8;
  const int iters = (nvec + kQuantThreads - 1) / kQuantThreads;
  float amax = 0.f;
  for (int it = 0; it < iters; ++it) {
    const int vec = it * kQuantThreads + threadIdx.x;
    float v[8];
    load_vec<T>(a, row, vec, vec < nvec, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x / 32] = amax;
  __syncthreads();
  amax = 0.f;
#pragma unroll
  for (int w = 0; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, warp_max[w]);
  const float inv = inv_scale(a, amax);
  if (threadIdx.x == 0) a.scales[row] = amax * a.inv_max_val;
  for (int it = 0; it < iters; ++it) {
    const int vec = it * kQuantThreads + threadIdx.x;
    float v[8];
    load_vec<T>(a, row, vec, vec < nvec, v);
    if (vec < nvec) {
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float q = fminf(fmaxf(rintf(v[i] * inv), -a.max_val), a.max_val);
        packed[i / 4] |= (uint32_t(int32_t(q)) & 0xFFu) << (8 * (i % 4));
      }
      *reinterpret_cast<uint2*>(a.xq + int64_t(row) * a.n + 8 * vec) = make_uint2(packed[0], packed[1]);
    }
  }
}

// Rows of at most kIters * kThreads * 8 elements: the row's raw bytes stay in
// registers between the max pass and the rounding pass, so it is read from
// memory once, with all of a thread's loads in flight together; the transform
// is recomputed for the rounding pass (the same operations in the same order
// as quant_rows_kernel, so the same bytes come out).
template <typename T, int kIters, int kThreads>
__global__ void __launch_bounds__(kThreads, 1024 / kThreads) quant_rows_reg_kernel(const QuantArgs a) {
  __shared__ float warp_max[kThreads / 32];
  griddep_wait();  // launched early behind the previous kernel (programmatic dependent launch)
  griddep_launch_dependents();
  const int row = blockIdx.x;
  const int nvec = a.n / 8;
  uint4 raw[kIters];
#pragma unroll
  for (int it = 0; it < kIters; ++it) {  // every load of the row in flight at once
    const int vec = it * kThreads + threadIdx.x;
    raw[it] = load_raw<T>(a, row, vec, vec < nvec);
  }
  float amax = 0.f;
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int vec = it * kThreads + threadIdx.x;
    float v[8];
    vec_from_raw<T>(a, row, vec, vec < nvec, raw[it], v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x / 32] = amax;
  __syncthreads();
  amax = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) amax = fmaxf(amax, warp_max[w]);
  const float inv = inv_scale(a, amax);
  if (threadIdx.x == 0) a.scales[row] = amax * a.inv_max_val;
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int vec = it * kThreads + threadIdx.x;
    float v[8];
    vec_from_raw<T>(a, row, vec, vec < nvec, raw[it], v);  // the same values again: no second read
    if (vec < nvec) {
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float q = fminf(fmaxf(rintf(v[i] * inv), -a.max_val), a.max_val);
        packed[i / 4] |= (uint32_t(int32_t(q)) & 0xFFu) << (8 * (i % 4));
      }
      *reinterpret_cast<uint2*>(a.xq + int64_t(row) * a.n + 8 * vec) = make_uint2(packed[0], packed[1]);
    }
  }
}

// Launched with programmatic stream serialization: the grid is scheduled
// while the previous kernel drains and waits for it in griddep_wait, and it
// lets the next kernel (the GEMM reading its output) start its own set-up.
template <typename K>
void launch_pdl(K kernel, int blocks, int threads, const QuantArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(blocks), 1, 1);
  cfg.blockDim = dim3(unsigned(threads), 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, a);
}

template <typename T>
void launch_quant(const QuantArgs& a, cudaStream_t s) {
  // Four 16-byte vectors per thread and 1024 resident threads per SM: 64 KB
  // of each SM's loads in flight whatever the row length.
  const int nvec = a.n / 8;
  if (nvec <= 256)
    launch_pdl(quant_rows_reg_kernel<T, 4, 64>, a.m, 64, a, s);
  else if (nvec <= 512)
    launch_pdl(quant_rows_reg_kernel<T, 4, 128>, a.m, 128, a, s);
  else if (nvec <= 1024)
    launch_pdl(quant_rows_reg_kernel<T, 4, 256>, a.m, 256, a, s);
  else if (nvec <= 2048)
    launch_pdl(quant_rows_reg_kernel<T, 4, 512>, a.m, 512, a, s);
  else
    launch_pdl(quant_rows_kernel<T>, a.m, kQuantThreads, a, s);
}

}  // namespace
}  // namespace pb2

extern "C" int pb2_quantize(const pb2_quant_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_quantize");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_quant_params& p = *pp;
  if (p.m < 0 || p.n <= 0 || p.m > INT32_MAX || p.n > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  if (!p.x || !p.xq || !p.scales || p.max_val <= 0 || p.max_val > 127) return PB2_ERR_INVALID_ARGUMENT;
  if (p.n % 8 != 0) return PB2_ERR_UNSUPPORTED_CONFIG;  // 16-byte row vectors
  if (p.block_size != 0) {
    const int k = p.block_size;
    // Blocks span whole 8-element vectors of one warp (the reference's
    // layout: hadamard.py:556-571).
    if (k < 8 || (k & (k - 1)) != 0 || k > 256 || p.n % k != 0) return PB2_ERR_UNSUPPORTED_CONFIG;
  }
  if (reinterpret_cast<uintptr_t>(p.x) % 16 || reinterpret_cast<uintptr_t>(p.xq) % 8 ||
      (p.smooth && reinterpret_cast<uintptr_t>(p.smooth) % 16))
    return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  if (p.m == 0) return PB2_OK;
  QuantArgs a;
  a.x = p.x;
  a.smooth = p.smooth;
  a.smooth_per_row = p.smooth_per_row;
  a.xq = p.xq;
  a.scales = p.scales;
  a.m = int(p.m);
  a.n = int(p.n);
  a.block = p.block_size;
  a.norm = p.block_size ? float(1.0 / sqrt(double(p.block_size))) : 1.0f;
  a.max_val = float(p.max_val);
  a.inv_max_val = float(1.0 / double(p.max_val));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.x_is_fp16)
    launch_quant<__half>(a, s);
  else
    launch_quant<__nv_bfloat16>(a, s);
  return launch_status();
}

namespace pb2 {
namespace {
__global__ void rcp_approx_kernel(const float* in, float* out, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = rcp_approx_ftz(in[i]);
}
}  // namespace
}  // namespace pb2

extern "C" int pb2_rcp_approx_f32(int device, const float* in, float* out, int64_t n, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_rcp_approx_f32");
  using namespace pb2;
  if (n < 0 || (n > 0 && (!in || !out))) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(device);
  if (st) return st;
  if (n == 0) return PB2_OK;
  const int blocks = int(std::min<int64_t>((n + 255) / 256, 4096));
  rcp_approx_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(in, out, n);
  return launch_status();
}
