// pb2_host.cu -- host-side helpers of the C ABI: tensor-map encoding through
// the driver entry point (no libcuda link dependency), device selection,
// status strings and the signalling-buffer sizes.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>

#include <nvtx3/nvToolsExt.h>

#include "pb2_common.cuh"

namespace pb2 {

namespace {
thread_local char g_last_cuda_error[256] = "";

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int note_cuda(cudaError_t e) {
  if (e == cudaSuccess) return PB2_OK;
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  return PB2_ERR_CUDA;
}
}  // namespace

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return PB2_ERR_NO_DRIVER_ENTRY;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return PB2_ERR_INVALID_ARGUMENT;
  if ((inner * elem_bytes) % 16 != 0) return PB2_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error),
                  "cuTensorMapEncodeTiled failed (%d)", int(r));
    return PB2_ERR_INVALID_ARGUMENT;
  }
  return PB2_OK;
}

// 3-D tiled map (dims inner, mid, outer; row-major, no padding): each
// dimension clips on its own, so a box never crosses into the next slab.
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t inner, uint64_t mid, uint64_t outer, uint32_t box_inner, uint32_t box_mid,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return PB2_ERR_NO_DRIVER_ENTRY;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return PB2_ERR_INVALID_ARGUMENT;
  if ((inner * elem_bytes) % 16 != 0) return PB2_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[3] = {inner, mid, outer};
  cuuint64_t strides[2] = {inner * elem_bytes, inner * mid * elem_bytes};
  cuuint32_t box[3] = {box_inner, box_mid, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error),
                  "cuTensorMapEncodeTiled failed (%d)", int(r));
    return PB2_ERR_INVALID_ARGUMENT;
  }
  return PB2_OK;
}

int set_device(int device) { return note_cuda(cudaSetDevice(device)); }

int sm_count(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 0;
  if (!cache[device]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) == cudaSuccess)
      cache[device] = v;
  }
  return cache[device];
}

int launch_status() { return note_cuda(cudaGetLastError()); }

namespace {
std::atomic<long long> g_wait_budget{PB2_DEFAULT_WAIT_BUDGET_CYCLES};
}  // namespace

long long wait_budget_cycles() { return g_wait_budget.load(std::memory_order_relaxed); }

// A minimal kernel that waits on mbarriers nobody arrives at: one warp with
// the spinning wait, one with the sleeping wait, each with the given budget.
// Both run out, record PB2_ERR_DEVICE_TIMEOUT in the sync word's error field
// and return; the kernel ends without any other effect.
__global__ void wait_selftest_kernel(SignalSync* sync, long long budget) {
  __shared__ uint64_t never[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&never[0], 1);
    mbar_init(&never[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int warp = threadIdx.x / 32;
  // A private abort flag per warp, so each warp's wait runs out on its own
  // clock rather than seeing the other's abort.
  volatile int mine = 0;
  bool ok;
  if (warp == 0)
    ok = mbar_wait_warp(&never[0], 0, &mine, sync, budget, suspend_hint_ns(budget));
  else
    ok = mbar_wait_idle_warp(&never[1], 0, &mine, sync, budget, suspend_hint_ns(budget));
  if (!ok && (threadIdx.x & 31) == 0) atomicAdd(&abort_flag, 1);
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag != 2) record_error(sync, PB2_ERR_INVALID_ARGUMENT);
}

int cuda_status(cudaError_t e) { return note_cuda(e); }

bool nvtx_enabled() {
  static const bool on = std::getenv("PEARL_B200_NVTX") != nullptr;
  return on;
}
NvtxRange::NvtxRange(const char* name) : on(nvtx_enabled()) {
  if (on) nvtxRangePushA(name);
}
NvtxRange::~NvtxRange() {
  if (on) nvtxRangePop();
}

}  // namespace pb2

extern "C" {

int64_t pb2_host_signal_header_size(void) { return PB2_HOST_SIGNAL_HEADER_SIZE; }
int64_t pb2_host_signal_sync_size(void) { return PB2_HOST_SIGNAL_SYNC_SIZE; }
int pb2_abi_version(void) { return PB2_ABI_VERSION; }

const char* pb2_status_string(int status) {
  switch (status) {
    case PB2_OK:
      return "ok";
    case PB2_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case PB2_ERR_UNSUPPORTED_CONFIG:
      return "no kernel found with given config";
    case PB2_ERR_CUDA:
      return "CUDA runtime error";
    case PB2_ERR_DEVICE_TIMEOUT:
      return "a device-side wait ran out of its budget";
    case PB2_ERR_NO_DRIVER_ENTRY:
      return "cuTensorMapEncodeTiled is not available from the driver";
    case PB2_ERR_SCRATCH_LIMIT:
      return "problem too large for the library's static scratch (PB2_STATIC_SCRATCH_BYTES)";
    default:
      return "unknown status";
  }
}

const char* pb2_last_cuda_error(void) { return pb2::g_last_cuda_error; }

int64_t pb2_set_wait_budget_cycles(int64_t cycles) {
  const long long v = cycles > 0 ? cycles : PB2_DEFAULT_WAIT_BUDGET_CYCLES;
  return pb2::g_wait_budget.exchange(v);
}

int pb2_wait_selftest(int device, int64_t budget_cycles, void* host_signal_sync, void* stream) {
  if (!host_signal_sync || budget_cycles <= 0 || budget_cycles > PB2_DEFAULT_WAIT_BUDGET_CYCLES)
    return PB2_ERR_INVALID_ARGUMENT;
  int st = pb2::set_device(device);
  if (st) return st;
  pb2::wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<pb2::SignalSync*>(host_signal_sync), budget_cycles);
  return pb2::launch_status();
}

}  // extern "C"
