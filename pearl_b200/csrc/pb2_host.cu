// pb2_host.cu -- host-side helpers of the C ABI: tensor-map encoding through
// the driver entry point (no libcuda link dependency), device selection,
// status strings and the signalling-buffer sizes.
#include <cstdio>
#include <cstring>
#include <mutex>

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

int cuda_status(cudaError_t e) { return note_cuda(e); }

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

}  // extern "C"
