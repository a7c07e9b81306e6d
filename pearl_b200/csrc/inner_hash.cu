// inner_hash.cu -- test aid mirroring the reference's inner_hash operator
// (miner/pearl-gemm/csrc/gemm/inner_hash_kernel.cu:11-58): the XOR of a
// 64..256-word buffer, added up `iterations` times.
#include "pb2_common.cuh"

namespace pb2 {
namespace {
__global__ void inner_hash_kernel(const uint32_t* __restrict__ in, int n, uint32_t* out,
                                  long long iterations) {
  // one warp: lane-strided XOR, butterfly reduction
  uint32_t x = 0;
  for (int i = threadIdx.x; i < n; i += 32) x ^= in[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x ^= __shfl_xor_sync(0xffffffffu, x, o);
  if (threadIdx.x == 0) {
    uint32_t acc = 0;
    for (long long i = 0; i < iterations; ++i) acc += x;
    *out = acc;
  }
}
}  // namespace
}  // namespace pb2

extern "C" int pb2_inner_hash(int device, const uint32_t* in, int64_t n, uint32_t* out,
                              int64_t iterations, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_inner_hash");
  using namespace pb2;
  if (!in || !out) return PB2_ERR_INVALID_ARGUMENT;
  if (!(n == 64 || n == 96 || n == 128 || n == 192 || n == 256)) return PB2_ERR_INVALID_ARGUMENT;
  if (!(iterations == 1 || iterations == 100000)) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(device);
  if (st) return st;
  inner_hash_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(in, int(n), out, iterations);
  return launch_status();
}
