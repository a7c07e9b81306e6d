// mma_tmem_contention.cu -- does loading TMEM slow the tensor core?  One CTA
// per SM: warp 0 streams kind::i8 M128 N256 K32 MMAs (cta_group::1) into TMEM
// columns [256, 512) in batches of 16 and times them; W other warps load
// columns [0, 256) with 32x32b.x32 (or two of them) until the MMA warp is done.
// Prints cycles per MMA and the readers' TMEM bytes per cycle per SM.
#include <cstdio>
#include <vector>
#include "../csrc/pb2_common.cuh"

using namespace pb2;

__global__ void bench(int n_batches, int readers, int x_per_iter, unsigned long long* out, uint32_t* sink) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t tbase;
  __shared__ uint64_t bar;
  __shared__ volatile int stop;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  if (threadIdx.x == 0) { mbar_init(&bar, 1); stop = 0; fence_barrier_init(); }
  // operand tiles: A 128 x 128 bytes at 0, B 256 x 128 bytes at 16 KB (SW128)
  for (int i = threadIdx.x; i < 48 * 1024 / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] = uint32_t(i) * 2654435761u;
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t t = tbase;
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t ad = sdesc_sw128(smem_u32(smem)), bd = sdesc_sw128(smem_u32(smem) + 16384);
      uint32_t ph = 0;
      const long long t0 = clock64();
      for (int b = 0; b < n_batches; ++b) {
        for (int j = 0; j < 16; ++j) umma_i8(t + 256, ad + 2 * (j & 3), bd + 2 * (j & 3), idesc_i8(128, 256), 1);
        umma_commit(&bar);
        const long long w0 = clock64();
        while (!mbar_test(&bar, ph) && clock64() - w0 < 200000000LL) {
        }
        ph ^= 1;
      }
      out[blockIdx.x] = clock64() - t0;
      stop = 1;
    }
  } else if (warp <= readers) {
    const int q = warp & 3;
    const uint32_t base = t + (uint32_t(32 * q) << 16) + (((warp - 1) / 4) * 64) % 256;
    uint32_t acc = 0;
    long long n = 0;
    const long long t0 = clock64();
    while (!stop && clock64() - t0 < 2000000000LL) {
      uint32_t v[64];
      tmem_ld32(base, v);
      if (x_per_iter == 64) tmem_ld32(base + 32, v + 32);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 64; ++i)
        if (i < x_per_iter) acc ^= v[i];  // constant indices: v stays in registers
      ++n;
    }
    sink[blockIdx.x * blockDim.x + threadIdx.x] = acc + uint32_t(n);
    if (lane == 0) atomicAdd(&out[gridDim.x + blockIdx.x], (unsigned long long)n);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) { __syncwarp(); tmem_dealloc(t, 512); }
}

int main() {
  const int sms = 148, nb = 400;
  unsigned long long* out;
  uint32_t* sink;
  cudaMalloc(&out, sizeof(unsigned long long) * sms * 2);
  cudaMalloc(&sink, sizeof(uint32_t) * sms * 32 * 20);
  cudaFuncSetAttribute(bench, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  for (int x : {32, 64}) {
    for (int r : {0, 4, 8, 12, 16}) {
      cudaMemset(out, 0, sizeof(unsigned long long) * sms * 2);
      bench<<<sms, 32 * (1 + r), 100 * 1024>>>(nb, r, x, out, sink);
      const cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); return 1; }
      std::vector<unsigned long long> h(sms * 2);
      cudaMemcpy(h.data(), out, sizeof(unsigned long long) * sms * 2, cudaMemcpyDeviceToHost);
      double cyc = 0, loads = 0;
      for (int b = 0; b < sms; ++b) { cyc += h[b]; loads += h[sms + b]; }
      cyc /= sms;
      loads /= sms;
      printf("x%d readers %2d: %.1f cycles per MMA, readers' TMEM %.0f B/cycle/SM\n", x, r, cyc / (nb * 16),
             loads * 32 * x * 4 / cyc);
    }
  }
  return 0;
}
