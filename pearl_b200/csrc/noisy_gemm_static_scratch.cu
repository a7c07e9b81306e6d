// noisy_gemm_static_scratch.cu -- pb2_noisy_gemm_static_scratch: the mined
// GEMM for callers that cannot allocate device memory.
//
// pb2_noisy_gemm's exact noising path needs two int32 scratch buffers from
// the caller (AxEBL_int32, EARxBpEB_int32): noise_A / noise_B add their
// split-K partial projections into them, and the converter turns them into
// the half factors the main kernel reads.  Some callers have no way to hand
// over such a buffer: a host that reaches this library only through its C
// ABI and has no device allocator of its own, or a process whose device
// memory belongs to another allocator (an inference server reserves most of
// HBM for its own pool when it starts, so an extra cudaMalloc can fail, and a
// cudaFree stalls every stream on the device).  This entry point keeps those
// two buffers in one fixed array of this file instead, so it allocates
// nothing at call time.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds PB2_STATIC_SCRATCH_BYTES of it until the process exits.  In
// host code its name only stands for the symbol; the device address comes
// from cudaGetSymbolAddress, looked up once per device (with that device
// current) on the first call there and cached.  That first call should come
// before any stream capture.  All calls on a device share the array and it
// keeps the last call's contents, so each call clears the words it uses
// before the noising kernels add into them, and calls that overlap on the
// GPU (different streams, no ordering between them) race on it.
#include <mutex>

#include "pb2_common.cuh"

namespace {

constexpr int64_t kScratchWords = PB2_STATIC_SCRATCH_BYTES / 4;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int32_t g_noising_scratch[kScratchWords];

std::mutex g_scratch_mutex;
int32_t* g_scratch_addr[kMaxDevices] = {};

// Device address of g_noising_scratch on `device`, which must be current.
int scratch_on(int device, int32_t** out) {
  if (device < 0 || device >= kMaxDevices) return PB2_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noising_scratch);
    if (e != cudaSuccess) return pb2::cuda_status(e);
    g_scratch_addr[device] = static_cast<int32_t*>(p);
  }
  *out = g_scratch_addr[device];
  return PB2_OK;
}

}  // namespace

extern "C" int pb2_noisy_gemm_static_scratch(const pb2_gemm_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_noisy_gemm_static_scratch");
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_gemm_params& p = *pp;
  // The int32 projections live in the library's array, never in the caller's.
  if (p.AxEBL_int32 || p.EARxBpEB_int32) return PB2_ERR_INVALID_ARGUMENT;
  if (p.m <= 0 || p.n <= 0 || p.r <= 0) return PB2_ERR_INVALID_ARGUMENT;
  if (p.m > kScratchWords || p.n > kScratchWords || p.r > kScratchWords) return PB2_ERR_SCRATCH_LIMIT;
  const int64_t a_words = p.run_noising_a ? p.m * p.r : 0;
  const int64_t b_words = p.run_noising_b ? p.n * p.r : 0;
  if (a_words + b_words > kScratchWords) return PB2_ERR_SCRATCH_LIMIT;

  // Every argument error is returned before the clear below is queued: a
  // rejected call must not touch the array an earlier call may still use.
  int st = pb2::check_noisy_gemm_args(p);
  if (st) return st;
  if ((st = pb2::set_device(p.device))) return st;
  int32_t* scratch = nullptr;
  if ((st = scratch_on(p.device, &scratch))) return st;
  pb2_gemm_params q = p;
  q.AxEBL_int32 = a_words ? scratch : nullptr;
  q.EARxBpEB_int32 = b_words ? scratch + a_words : nullptr;
  if (a_words + b_words > 0) {
    const cudaError_t e = cudaMemsetAsync(scratch, 0, size_t(a_words + b_words) * sizeof(int32_t),
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return pb2::cuda_status(e);
  }
  return pb2_noisy_gemm(&q, stream);
}
