// scatter.cu -- row scatter of the mined MoE layer.
//
// The MoE GEMM1 writes each expert's rows in expert order and puts them back
// in routing-slot order (miner/vllm-miner/src/vllm_miner/pearl_moe_experts.py:
// 347, cache_flat[expert_slot_indices] = expert_output).  One block per
// source row copies it with 16-byte loads and stores: both sides coalesced,
// so the scatter runs at HBM speed.
#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) scatter_rows_kernel(const uint4* __restrict__ src,
                                                                uint4* __restrict__ dst,
                                                                const int32_t* __restrict__ idx,
                                                                int64_t dst_rows, int64_t row_vec) {
  const int64_t r = blockIdx.x;
  const int32_t d = idx[r];
  if (d < 0 || d >= dst_rows) return;
  const uint4* s = src + r * row_vec;
  uint4* o = dst + int64_t(d) * row_vec;
  for (int64_t i = threadIdx.x; i < row_vec; i += kThreads) o[i] = s[i];
}

}  // namespace
}  // namespace pb2

extern "C" int pb2_scatter_rows(const pb2_scatter_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_scatter_rows");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_scatter_params& p = *pp;
  if (!p.src || !p.dst || !p.indices) return PB2_ERR_INVALID_ARGUMENT;
  if (p.rows < 0 || p.dst_rows < 0 || p.row_bytes <= 0 || p.row_bytes % 16 != 0) return PB2_ERR_INVALID_ARGUMENT;
  if (p.rows > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(p.src) % 16 || reinterpret_cast<uintptr_t>(p.dst) % 16)
    return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  if (p.rows == 0) return PB2_OK;
  scatter_rows_kernel<<<unsigned(p.rows), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(p.src), static_cast<uint4*>(p.dst), p.indices, p.dst_rows, p.row_bytes / 16);
  return launch_status();
}
