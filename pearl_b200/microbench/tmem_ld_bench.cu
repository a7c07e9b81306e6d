// tmem_ld_bench.cu -- TMEM load microbenchmark: throughput of tcgen05.ld
// 32x32b.xN and 16x256b.x8 with W warps per CTA, optionally with an MMA warp
// streaming into the other half of TMEM.  One CTA per SM.
#include <cstdio>
#include <cstdlib>
#include <vector>
#include "../csrc/pb2_common.cuh"

using namespace pb2;

// SHAPE 0: X columns of 32x32b (thread = lane); SHAPE 1: X / 32 loads of
// 16x256b.x8 (16 lanes x 64 columns each, the same 4 KB per load per warp).
template <int X, int SHAPE>
__device__ __forceinline__ void ldx(uint32_t taddr, uint32_t* v) {
#pragma unroll
  for (int i = 0; i < X / 32; ++i) {
    if (SHAPE == 0) tmem_ld32(taddr + 32 * i, v + 32 * i);
    else tmem_ld16x256_x8(taddr + 64 * i, v + 32 * i);
  }
}

template <int X, int SHAPE>
__global__ void bench(int iters, int mma_on, unsigned long long* out, uint32_t* sink) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tbase;
  __shared__ uint64_t bar;
  __shared__ int done_count;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nw = blockDim.x / 32;
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  if (threadIdx.x == 0) { mbar_init(&bar, 1); done_count = 0; fence_barrier_init(); }
  // zero smem operands
  for (int i = threadIdx.x; i < 48 * 1024 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(smem)[i] = 0;
  asm volatile("fence.proxy.async.shared::cta;");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  uint32_t t = tbase;
  if (warp == nw - 1 && mma_on) {
    // MMA warp: stream kind::i8 MMAs into columns [256, 512)
    if (lane == 0) {
      uint64_t ad = sdesc_sw128(smem_u32(smem)), bd = sdesc_sw128(smem_u32(smem) + 16384);
      uint32_t ph = 0;
      long long n = 0;
      const int readers = nw - 1;
      long long tstart = clock64();
      while (atomicAdd(&done_count, 0) < readers && clock64() - tstart < 2000000000LL) {
        for (int j = 0; j < 64; ++j) umma_i8(t + 256, ad + 2 * (j & 3), bd + 2 * (j & 3), idesc_i8(128, 256), 1);
        umma_commit(&bar);
        long long w0 = clock64();
        while (!mbar_test(&bar, ph) && clock64() - w0 < 200000000LL) {}
        ph ^= 1;
        n += 64;
      }
      out[gridDim.x * 64 + blockIdx.x] = n;
    }
  } else if (warp < nw - (mma_on ? 1 : 0)) {
    const int q = warp & 3;
    const int slot = warp / 4;  // spread warps over columns
    uint32_t acc = 0;
    const uint32_t base = SHAPE == 0 ? t + (uint32_t(32 * q) << 16) + (slot * X) % 256
                                     : t + (uint32_t(32 * q + 16 * (slot & 1)) << 16) + ((slot >> 1) * 2 * X) % 256;
    __syncwarp();
    long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
      uint32_t v[X];
      ldx<X, SHAPE>(base, v);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < X; ++i) acc ^= v[i];
    }
    long long t1 = clock64();
    if (lane == 0) { out[blockIdx.x * 64 + warp] = t1 - t0; atomicAdd(&done_count, 1); }
    sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) { __syncwarp(); tmem_dealloc(t, 512); }
}

template <int X, int SHAPE = 0>
void run(int warps, int mma_on, int sms) {
  int threads = 32 * (warps + (mma_on ? 1 : 0));
  int iters = 2000;
  unsigned long long* out; uint32_t* sink;
  cudaMalloc(&out, sizeof(unsigned long long) * sms * 65 + 64);
  cudaMalloc(&sink, sizeof(uint32_t) * sms * threads);
  cudaMemset(out, 0, sizeof(unsigned long long) * sms * 65 + 64);
  cudaFuncSetAttribute(bench<X, SHAPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  bench<X, SHAPE><<<sms, threads, 100 * 1024>>>(iters, mma_on, out, sink);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); exit(1); }
  std::vector<unsigned long long> h(sms * 65);
  cudaMemcpy(h.data(), out, sizeof(unsigned long long) * sms * 65, cudaMemcpyDeviceToHost);
  double cyc = 0; int cnt = 0;
  for (int b = 0; b < sms; ++b) for (int w = 0; w < warps; ++w) { cyc += h[b * 64 + w]; cnt++; }
  cyc /= cnt;
  double per_iter = cyc / iters;
  double bytes_per_cycle = double(warps) * 32 * X * 4 / per_iter;
  printf("%s x%-3d warps %2d mma %d: %.1f cycles/iter/warp, %.0f B/cycle/SM\n", SHAPE ? "16x256b" : "32x32b ", X, warps, mma_on, per_iter, bytes_per_cycle);
  cudaFree(out); cudaFree(sink);
}

int main(int argc, char** argv) {
  int sms = 148;
  if (argc > 1) {  // 16x256b shape only
    for (int mma = 0; mma < 2; ++mma)
      for (int w : {4, 8, 16}) {
        run<32, 0>(w, mma, sms);
        run<32, 1>(w, mma, sms);
        run<64, 1>(w, mma, sms);
      }
    return 0;
  }
  for (int mma = 0; mma < 2; ++mma) {
    for (int w : {4, 8, 16}) {
      run<32>(w, mma, sms);
      run<64>(w, mma, sms);
      if (w <= 8) run<128>(w, mma, sms);
    }
  }
  return 0;
}
