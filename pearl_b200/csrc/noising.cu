// noising.cu -- operand noising and denoise-factor projection on tcgen05.
//
// Semantics of the reference operators noise_A / noise_B
// (miner/pearl-gemm/csrc/gemm/pearl_gemm_api.cpp:300-500, kernels
// pearl_noisingA_kernel.h / pearl_noisingB_kernel.h, docstrings in
// src/pearl_gemm/pearl_gemm_interface.py:122-230), exact for any int8
// factor matrices:
//   XpE  = int8(X + EL . E_rmajor^T)       (EA = EAL . EAR, EB = EBR . EBL)
//   proj = Xs . E_kmajor^T                 (Xs = X for noise_A, XpE for noise_B)
// One CTA owns 128 rows of X and a range of 128-wide k-blocks.  Per k-block
// the MMA warp computes D1 = EL . E_rmajor[kb]^T (128 x 128 int32, K = r) into
// one of two TMEM slots and accumulates D2 += Xs[kb] . E_kmajor[kb]^T
// (128 x r int32); four epilogue warps (thread = row) add X from the TMA'd
// shared-memory tile, store XpE and -- for noise_B -- write the noised tile
// back into shared memory in the UMMA operand layout so the projection reads
// the noised values.  The projection is written as half (x 2^-14 for AxEBL,
// x 2^-12 for EARxBpEB) or accumulated into int32 (the caller zeroes it, as
// the reference's split-K path requires).  With half output and a K split,
// the CTAs of one row block form a cluster and rank 0 sums the int32 partials
// from its peers' shared memory before converting, so no global scratch is
// used.
#include <algorithm>
#include <cstring>

#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int NM = 128;  // rows of X per CTA
constexpr int NKB = 128; // k per k-block
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
constexpr int kStages = 3;
constexpr int kElBytes = 16 * 1024;
constexpr int kStageSlot = 48 * 1024;  // X 16 KB + E_rmajor tile + E_kmajor tile
constexpr int kXpBytes = 16 * 1024;
constexpr int kSmemPlan = kElBytes + kStages * kStageSlot + 2 * kXpBytes;

struct NoisingArgs {
  CUtensorMap tmX, tmEL, tmE1, tmE2;
  int rows, K, nkb, kbps, ks;
  int use_cluster;
  int proj_fp16;
  float scale;
  int8_t* XpE;
  void* proj;
  SignalSync* sync;
};

struct NSmem {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t el_full;
  uint64_t d1_full[2];
  uint64_t d1_empty[2];
  uint64_t xp_full[2];
  uint64_t xp_empty[2];
  uint64_t d2_full;
  uint64_t red_ready;
  uint64_t red_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ bool wait_cluster_bounded(uint64_t* bar, uint32_t parity) {
  long long t0 = clock64();
  while (!mbar_test_cluster(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles) return false;
  }
  return true;
}

// Byte offset of 16-byte chunk `ch` of row `row` in a 128-byte-row tile with
// the 128-byte swizzle (the layout TMA writes and UMMA reads).
__device__ __forceinline__ uint32_t sw128_off(int row, int ch) {
  return uint32_t(row) * 128u + (uint32_t(ch ^ (row & 7)) << 4);
}

template <int R, bool kB>
__global__ void __launch_bounds__(kThreads, 1) noising_kernel(const __grid_constant__ NoisingArgs a) {
  constexpr int kE1Bytes = NKB * R;
  constexpr int kE2Bytes = R * NKB;
  constexpr uint32_t kTxBytes = NM * NKB + kE1Bytes + kE2Bytes;
  constexpr uint32_t kIdesc1 = idesc_i8(NM, NKB);
  constexpr uint32_t kIdesc2 = idesc_i8(NM, R);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* el_buf = base;
  uint8_t* stages = base + kElBytes;
  uint8_t* xp_buf = stages + kStages * kStageSlot;
  NSmem& S = *reinterpret_cast<NSmem*>(base + kSmemPlan);
  volatile int* abort_flag = &S.abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb0 = blockIdx.y * a.kbps;
  const int nkb = min(a.kbps, a.nkb - kb0);
  const int r0 = blockIdx.x * NM;
  const uint32_t rank = a.use_cluster ? cluster_ctarank() : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], 1 + 4);
    }
    mbar_init(&S.el_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.d1_full[i], 1);
      mbar_init(&S.d1_empty[i], 4);
      mbar_init(&S.xp_full[i], 4);
      mbar_init(&S.xp_empty[i], 1);
    }
    mbar_init(&S.d2_full, 1);
    mbar_init(&S.red_ready, a.use_cluster ? 4 * (a.ks - 1) : 1);
    mbar_init(&S.red_done, 4);
    mbar_init(&S.drain, 1);
    S.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&S.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (a.use_cluster) cluster_sync_all();  // peers' barriers are initialized
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch(&a.tmX);
      tma_prefetch(&a.tmE1);
      tma_prefetch(&a.tmE2);
      mbar_arrive_expect_tx(&S.el_full, NM * R);
      tma_load_2d(&a.tmEL, &S.el_full, el_buf, 0, r0);
      int i = 0;
      for (; i < nkb; ++i) {
        const int s = i % kStages;
        if (!mbar_wait(&S.empty[s], ((i / kStages) & 1) ^ 1, abort_flag, a.sync)) break;
        mbar_arrive_expect_tx(&S.full[s], kTxBytes);
        uint8_t* st = stages + s * kStageSlot;
        const int k = (kb0 + i) * NKB;
        tma_load_2d(&a.tmX, &S.full[s], st, k, r0);
        tma_load_2d(&a.tmE1, &S.full[s], st + 16384, 0, k);
        tma_load_2d(&a.tmE2, &S.full[s], st + 32768, k, 0);
      }
      for (int j = (i > kStages ? i - kStages : 0); j < i; ++j) {
        long long t0 = clock64();
        while (!mbar_test(&S.full[j % kStages], (j / kStages) & 1) && clock64() - t0 < 100000000LL) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&S.el_full, 0, abort_flag, a.sync);
      const uint32_t el = smem_u32(el_buf);
      auto mma2_b = [&](int j) -> bool {
        const int ps = j & 1;
        if (!mbar_wait(&S.xp_full[ps], (j >> 1) & 1, abort_flag, a.sync)) return false;
        tc_fence_after();
        const uint64_t ad = sdesc_kmajor<128>(smem_u32(xp_buf + ps * kXpBytes));
        const uint64_t bd = sdesc_kmajor<128>(smem_u32(stages + (j % kStages) * kStageSlot + 32768));
#pragma unroll
        for (int ks = 0; ks < NKB / 32; ++ks) umma_i8(tmem + 256, ad + 2 * ks, bd + 2 * ks, kIdesc2, (j | ks) != 0);
        umma_commit(&S.xp_empty[ps]);
        umma_commit(&S.empty[j % kStages]);
        return true;
      };
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % kStages, slot = i & 1;
        if (!(ok = mbar_wait(&S.full[s], (i / kStages) & 1, abort_flag, a.sync))) break;
        if (i >= 2 && !(ok = mbar_wait(&S.d1_empty[slot], ((i >> 1) - 1) & 1, abort_flag, a.sync))) break;
        tc_fence_after();
        const uint32_t st = smem_u32(stages + s * kStageSlot);
        {
          const uint64_t ad = sdesc_kmajor<R>(el);
          const uint64_t bd = sdesc_kmajor<R>(st + 16384);
#pragma unroll
          for (int ks = 0; ks < R / 32; ++ks) umma_i8(tmem + 128 * slot, ad + 2 * ks, bd + 2 * ks, kIdesc1, ks != 0);
          umma_commit(&S.d1_full[slot]);
        }
        if (!kB) {
          const uint64_t ad = sdesc_kmajor<128>(st);
          const uint64_t bd = sdesc_kmajor<128>(st + 32768);
#pragma unroll
          for (int ks = 0; ks < NKB / 32; ++ks) umma_i8(tmem + 256, ad + 2 * ks, bd + 2 * ks, kIdesc2, (i | ks) != 0);
          umma_commit(&S.empty[s]);
        } else if (i >= 1) {
          ok = mma2_b(i - 1);
        }
      }
      if (ok && kB && nkb >= 1) ok = mma2_b(nkb - 1);
      umma_commit(&S.d2_full);
      umma_commit(&S.drain);
      long long t0 = clock64();
      while (!mbar_test(&S.drain, 0) && clock64() - t0 < 100000000LL) {
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = 32 * q + lane;  // row of the CTA tile this thread owns
    const int64_t grow = int64_t(r0) + row;
    const uint32_t trow = tmem + (uint32_t(32 * q) << 16);
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      const int s = i % kStages, slot = i & 1;
      if (!(ok = mbar_wait(&S.d1_full[slot], (i >> 1) & 1, abort_flag, a.sync))) break;
      // Also observe the stage's TMA completion: makes the X tile visible here.
      if (!(ok = mbar_wait(&S.full[s], (i / kStages) & 1, abort_flag, a.sync))) break;
      if (kB && i >= 2 && !(ok = mbar_wait(&S.xp_empty[slot], ((i >> 1) - 1) & 1, abort_flag, a.sync))) break;
      tc_fence_after();
      const uint8_t* xt = stages + s * kStageSlot;
      uint8_t* xp = xp_buf + slot * kXpBytes;
      const int64_t kcol0 = int64_t(kb0 + i) * NKB;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(trow + 128 * slot + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int ch = 2 * c + h;
          const uint4 xv = *reinterpret_cast<const uint4*>(xt + sw128_off(row, ch));
          const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
          uint32_t ow[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t o = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const int xb = int(int8_t((xw[w] >> (8 * b)) & 0xFF));
              const int val = xb + int(v[16 * h + 4 * w + b]);
              o |= (uint32_t(val) & 0xFFu) << (8 * b);
            }
            ow[w] = o;
          }
          const uint4 out = make_uint4(ow[0], ow[1], ow[2], ow[3]);
          const int64_t kc = kcol0 + 16 * ch;
          if (grow < a.rows && kc < a.K)
            *reinterpret_cast<uint4*>(a.XpE + grow * a.K + kc) = out;
          if (kB) *reinterpret_cast<uint4*>(xp + sw128_off(row, ch)) = out;
        }
      }
      __syncwarp();
      tc_fence_before();
      if (kB) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&S.d1_empty[slot]);
        mbar_arrive(&S.empty[s]);
        if (kB) mbar_arrive(&S.xp_full[slot]);
      }
    }
    // ---- projection: D2 (128 x R int32) -> proj
    if (ok) ok = mbar_wait(&S.d2_full, 0, abort_flag, a.sync);
    if (ok) {
      tc_fence_after();
      // The partial reuses the operand ring: wait until all four epilogue
      // warps are done reading their last X tile from it.
      if (a.use_cluster && rank != 0) named_barrier_sync(1, 128);
      int32_t* red = reinterpret_cast<int32_t*>(stages);  // the ring is idle now
      constexpr int kRedStride = R + 4;                   // words; 16-byte aligned rows
      const bool to_peer = a.use_cluster && rank != 0;
#pragma unroll 1
      for (int c = 0; c < R; c += 32) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(trow + 256 + c, v);
        tmem_wait_ld();
        if (to_peer) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<int4*>(red + row * kRedStride + c + j) =
                make_int4(int(v[j]), int(v[j + 1]), int(v[j + 2]), int(v[j + 3]));
          continue;
        }
        if (a.use_cluster) {
          // rank 0: add the peers' partials (published below) before converting
          if (c == 0) {
            __syncwarp();
            if (!wait_cluster_bounded(&S.red_ready, 0)) { ok = false; }
          }
          if (ok) {
            for (int r = 1; r < a.ks; ++r) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const int4 pv = ld_cluster_v4(mapa(red + row * kRedStride + c + j, uint32_t(r)));
                v[j] += uint32_t(pv.x); v[j + 1] += uint32_t(pv.y);
                v[j + 2] += uint32_t(pv.z); v[j + 3] += uint32_t(pv.w);
              }
            }
          }
        }
        if (grow < a.rows) {
          if (a.proj_fp16) {
            __half* o = static_cast<__half*>(a.proj) + grow * R + c;
#pragma unroll
            for (int j = 0; j < 32; j += 2)
              *reinterpret_cast<__half2*>(o + j) =
                  __floats2half2_rn(float(int(v[j])) * a.scale, float(int(v[j + 1])) * a.scale);
          } else {
            int* o = static_cast<int*>(a.proj) + grow * R + c;
#pragma unroll
            for (int j = 0; j < 32; ++j) atomicAdd(o + j, int(v[j]));
          }
        }
      }
      if (a.use_cluster) {
        __syncwarp();
        if (rank != 0) {
          // publish the partial to rank 0, then stay resident until it has read it
          if (lane == 0) mbar_arrive_remote(mapa(&S.red_ready, 0));
          if (!wait_cluster_bounded(&S.red_done, 0)) ok = false;
        } else if (lane == 0) {
          for (int r = 1; r < a.ks; ++r) mbar_arrive_remote(mapa(&S.red_done, uint32_t(r)));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

template <int R, bool kB>
int launch_noising(const NoisingArgs& a, int row_blocks, cudaStream_t s) {
  auto kern = noising_kernel<R, kB>;
  const int smem = kSmemPlan + int(sizeof(NSmem)) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(row_blocks), unsigned(a.ks), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (a.use_cluster) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = unsigned(a.ks);
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaLaunchKernelEx(&cfg, kern, a);
  return launch_status();
}

int run_noising(const pb2_noising_params& p, bool b_side, cudaStream_t stream) {
  if (!p.X || !p.EL || !p.E_rmajor || !p.E_kmajor || !p.XpE || !p.proj)
    return PB2_ERR_INVALID_ARGUMENT;
  if (p.rows <= 0 || p.k <= 0 || p.k % 16 != 0) return PB2_ERR_INVALID_ARGUMENT;
  if (p.rows > INT32_MAX || p.k > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  if (!(p.r == 64 || p.r == 128)) return PB2_ERR_UNSUPPORTED_CONFIG;
  const void* ptrs[] = {p.X, p.EL, p.E_rmajor, p.E_kmajor, p.XpE, p.proj};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) % 16) return PB2_ERR_INVALID_ARGUMENT;
  if (p.proj_is_fp16 && p.k_blocks_per_split > 0) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  const int r = int(p.r);
  const CUtensorMapSwizzle rswz = r == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  NoisingArgs a;
  std::memset(&a, 0, sizeof(a));
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if ((st = make_tmap_2d(&a.tmX, p.X, U8, 1, p.k, p.rows, NKB, NM, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (st = make_tmap_2d(&a.tmEL, p.EL, U8, 1, r, p.rows, r, NM, rswz)) ||
      (st = make_tmap_2d(&a.tmE1, p.E_rmajor, U8, 1, r, p.k, r, NKB, rswz)) ||
      (st = make_tmap_2d(&a.tmE2, p.E_kmajor, U8, 1, p.k, r, NKB, r, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  const int row_blocks = int((p.rows + NM - 1) / NM);
  const int nkb = int((p.k + NKB - 1) / NKB);
  const int sms = std::max(1, sm_count(p.device));
  int ks;
  if (p.proj_is_fp16) {
    // K split over a cluster (<= 8 CTAs) so that one wave covers the GPU.
    ks = std::max(1, std::min({8, nkb, sms / row_blocks}));
  } else if (p.k_blocks_per_split > 0) {
    ks = (nkb + p.k_blocks_per_split - 1) / p.k_blocks_per_split;
  } else if (p.k_blocks_per_split == 0) {
    ks = 1;
  } else {
    ks = std::max(1, std::min(nkb, (sms + row_blocks - 1) / row_blocks));
  }
  a.kbps = (nkb + ks - 1) / ks;
  a.ks = (nkb + a.kbps - 1) / a.kbps;
  a.use_cluster = p.proj_is_fp16 && a.ks > 1;
  a.rows = int(p.rows);
  a.K = int(p.k);
  a.nkb = nkb;
  a.proj_fp16 = p.proj_is_fp16;
  a.scale = b_side ? (1.0f / 4096.0f) : (1.0f / 16384.0f);
  a.XpE = p.XpE;
  a.proj = p.proj;
  a.sync = static_cast<SignalSync*>(p.host_signal_sync);
  if (r == 128) return b_side ? launch_noising<128, true>(a, row_blocks, stream)
                              : launch_noising<128, false>(a, row_blocks, stream);
  return b_side ? launch_noising<64, true>(a, row_blocks, stream)
                : launch_noising<64, false>(a, row_blocks, stream);
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
