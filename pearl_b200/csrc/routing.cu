// routing.cu -- build_routing_data on sm_100a: the canonical per-expert token
// order a mined MoE layer commits to (miner/pearl-gemm/csrc/moe/
// build_routing_data.cu:40-144, which runs a CUB radix sort).
//
// For the (m, top_k) expert ids, slot_indices lists the flat slot indices
// stably sorted by expert id (8-bit keys), routing_data = slot_indices /
// top_k (the token of each slot), and routing_offsets[e] = the number of
// slots whose expert id is <= e (exclusive segment ends).
//
// A stable counting sort in three launches over blocks of 8192 slots:
// per-block 256-bin histograms (shared-memory atomics), one CTA that turns
// them into each block's first output position per bin (bin-major scan, which
// is what makes the sort stable across blocks), and a scatter in which every
// block walks its slots in index order, 1024 at a time: __match_any_sync
// ranks equal keys inside a warp and a per-bin prefix over the 32 warps ranks
// them across the warps of the round.  The scratch holds the block x bin
// table (4 bytes each).
#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int kBins = 256;
constexpr int kSortThreads = 1024;
constexpr int kSlotsPerThread = 8;
constexpr int kBlockSlots = kSortThreads * kSlotsPerThread;

struct RoutingArgs {
  const int32_t* ids;
  int32_t* routing_data;
  int32_t* slot_indices;
  int32_t* offsets;
  int32_t* table;  // blocks x kBins
  int numel, top_k, num_experts, blocks;
};

__global__ void __launch_bounds__(kSortThreads) routing_count_kernel(const RoutingArgs a) {
  __shared__ int32_t hist[kBins];
  const int t = threadIdx.x;
  if (t < kBins) hist[t] = 0;
  __syncthreads();
  const int first = blockIdx.x * kBlockSlots;
  for (int i = t; i < kBlockSlots; i += kSortThreads) {
    const int idx = first + i;
    if (idx < a.numel) atomicAdd(&hist[a.ids[idx] & (kBins - 1)], 1);
  }
  __syncthreads();
  if (t < kBins) a.table[blockIdx.x * kBins + t] = hist[t];
}

__global__ void __launch_bounds__(kBins) routing_scan_kernel(const RoutingArgs a) {
  __shared__ int32_t total[kBins];
  __shared__ int32_t start[kBins];
  const int b = threadIdx.x;
  int run = 0;
  for (int blk = 0; blk < a.blocks; ++blk) {  // block starts within bin b
    const int c = a.table[blk * kBins + b];
    a.table[blk * kBins + b] = run;
    run += c;
  }
  total[b] = run;
  __syncthreads();
  if (b == 0) {
    int s = 0;
    for (int i = 0; i < kBins; ++i) {
      start[i] = s;
      s += total[i];
    }
  }
  __syncthreads();
  for (int blk = 0; blk < a.blocks; ++blk) a.table[blk * kBins + b] += start[b];
  if (b < a.num_experts) a.offsets[b] = start[b] + total[b];
}

__global__ void __launch_bounds__(kSortThreads) routing_scatter_kernel(const RoutingArgs a) {
  __shared__ int32_t next[kBins];             // this block's next output slot per bin
  __shared__ int32_t warp_count[32][kBins];   // per-warp counts, then per-warp starts
  const int t = threadIdx.x;
  const int warp = t / 32, lane = t % 32;
  if (t < kBins) next[t] = a.table[blockIdx.x * kBins + t];
  const int first = blockIdx.x * kBlockSlots;
  for (int r = 0; r < kSlotsPerThread; ++r) {
    for (int i = t; i < 32 * kBins; i += kSortThreads) (&warp_count[0][0])[i] = 0;
    __syncthreads();
    const int idx = first + r * kSortThreads + t;  // (warp, lane) order is index order
    const bool valid = idx < a.numel;
    const int key = valid ? (a.ids[idx] & (kBins - 1)) : -1;
    const unsigned same = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(same & ((1u << lane) - 1u));
    if (valid && lane == __ffs(same) - 1) warp_count[warp][key] = __popc(same);
    __syncthreads();
    int round_total = 0;
    if (t < kBins) {
      for (int w = 0; w < 32; ++w) {
        const int c = warp_count[w][t];
        warp_count[w][t] = round_total;
        round_total += c;
      }
    }
    __syncthreads();
    if (valid) {
      const int pos = next[key] + warp_count[warp][key] + rank;
      a.slot_indices[pos] = idx;
      a.routing_data[pos] = idx / a.top_k;
    }
    __syncthreads();
    if (t < kBins) next[t] += round_total;
  }
}

}  // namespace
}  // namespace pb2

extern "C" int64_t pb2_build_routing_data_scratchpad_bytes(int64_t numel) {
  if (numel <= 0) return 0;
  const int64_t blocks = (numel + pb2::kBlockSlots - 1) / pb2::kBlockSlots;
  return blocks * pb2::kBins * int64_t(sizeof(int32_t));
}

extern "C" int pb2_build_routing_data(const pb2_routing_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_build_routing_data");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_routing_params& p = *pp;
  if (p.num_tokens < 0 || p.top_k <= 0 || p.num_experts <= 0) return PB2_ERR_INVALID_ARGUMENT;
  if (p.num_experts > kBins) return PB2_ERR_INVALID_ARGUMENT;  // 8-bit expert ids
  const int64_t numel = p.num_tokens * p.top_k;
  if (numel > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  if (!p.routing_offsets || (numel > 0 && (!p.topk_ids || !p.routing_data || !p.slot_indices)))
    return PB2_ERR_INVALID_ARGUMENT;
  const int64_t need = pb2_build_routing_data_scratchpad_bytes(numel);
  if (numel > 0 && (!p.scratchpad || p.scratchpad_bytes < need || reinterpret_cast<uintptr_t>(p.scratchpad) % 4))
    return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (numel == 0) return cuda_status(cudaMemsetAsync(p.routing_offsets, 0, size_t(p.num_experts) * 4, s));
  RoutingArgs a;
  a.ids = p.topk_ids;
  a.routing_data = p.routing_data;
  a.slot_indices = p.slot_indices;
  a.offsets = p.routing_offsets;
  a.table = static_cast<int32_t*>(p.scratchpad);
  a.numel = int(numel);
  a.top_k = int(p.top_k);
  a.num_experts = int(p.num_experts);
  a.blocks = int((numel + kBlockSlots - 1) / kBlockSlots);
  routing_count_kernel<<<a.blocks, kSortThreads, 0, s>>>(a);
  if ((st = launch_status())) return st;
  routing_scan_kernel<<<1, kBins, 0, s>>>(a);
  if ((st = launch_status())) return st;
  routing_scatter_kernel<<<a.blocks, kSortThreads, 0, s>>>(a);
  return launch_status();
}
