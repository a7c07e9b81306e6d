// noising.cu -- operand noising and denoise-factor projection on tcgen05.
//
// Semantics of the reference operators noise_A / noise_B
// (miner/pearl-gemm/csrc/gemm/pearl_gemm_api.cpp:300-500, kernels
// pearl_noisingA_kernel.h / pearl_noisingB_kernel.h, docstrings in
// src/pearl_gemm/pearl_gemm_interface.py:122-230), exact for any int8
// factor matrices:
//   XpE  = int8(X + EL . E_rmajor^T)       (EA = EAL . EAR, EB = EBR . EBL)
//   proj = Xs . E_kmajor^T                 (Xs = X for noise_A, XpE for noise_B)
// One CTA owns nm <= 256 rows of X and a range of 128-wide k-blocks (rows of
// the 256-row MMA tile past nm hold stale shared memory: they are computed
// and never stored).  Per k-block
// the MMA warp computes D1 = EL . E_rmajor[kb]^T (256 x 128 int32, K = r, as
// two 128-row MMAs sharing the E tile) into TMEM and accumulates
// D2 += Xs[kb] . E_kmajor[kb]^T (256 x r int32).  Sixteen epilogue warps add
// the low bytes of D1 into the TMA'd X tile in shared memory, in place and
// four bytes per instruction, so the tile becomes the XpE tile in the same
// swizzled layout: the warps store it from there and, for noise_B, the
// projection MMA reads it from there.  The projection is written as half
// (x 2^-14 for AxEBL, x 2^-12 for EARxBpEB) or accumulated into int32 (the
// caller zeroes it, as the reference's split-K path requires).  With half
// output and a K split, the CTAs of one row block form a cluster; each
// stages its int32 partial in shared memory and each sums a slice of the
// rows over all of them (distributed shared memory), so no global scratch is
// used.
#include <algorithm>
#include <cstring>

#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int NM = 256;  // most rows of X per CTA (two 128-row MMA halves); NoisingArgs::nm <= NM
constexpr int NKB = 128; // k per k-block
constexpr int kEpiWarps = 16;  // per TMEM lane quadrant: 2 row halves x 2 column halves
constexpr int kThreads = 32 * (2 + kEpiWarps);  // TMA, MMA, 8 epilogue
constexpr int kStages = 3;
constexpr int kElBytes = NM * 128;               // EL rows, r <= 128 bytes each
constexpr int kXBytes = NM * NKB;                // X (then XpE) tile of a stage
constexpr int kStageSlot = kXBytes + 2 * 16384;  // + E_rmajor tile + E_kmajor tile
constexpr int kSmemPlan = kElBytes + kStages * kStageSlot;

struct NoisingArgs {
  CUtensorMap tmX, tmEL, tmE1, tmE2;
  int rows, K, nkb, kbps, ks;
  int nm;  // rows of X per CTA: a multiple of 8, at most NM (the TMA boxes of X and EL are nm rows high)
  int use_cluster;
  int proj_fp16;
  float scale;
  int8_t* XpE;
  void* proj;
  SignalSync* sync;
  long long wait_budget;  // SM cycles a device-side wait may spin (pb2_set_wait_budget_cycles)
};

struct NSmem {
  uint64_t full_e[kStages];   // E tiles of the stage landed
  uint64_t full_x[kStages];   // X tile of the stage landed
  uint64_t x_free[kStages];   // noise_A: the projection has read X
  uint64_t empty[kStages];
  uint64_t xp_ready[kStages];
  uint64_t el_full;
  uint64_t d1_full;
  uint64_t d1_empty;
  uint64_t d2_full;
  uint64_t red_ready;
  uint64_t red_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// Cluster-scope wait with one verdict for the whole warp (the callers go on
// to warp-wide code).
__device__ __forceinline__ bool wait_cluster_bounded(uint64_t* bar, uint32_t parity, long long budget) {
  long long t0 = clock64();
  bool ok = true;
  while (!mbar_test_cluster(bar, parity)) {
    if (clock64() - t0 > budget) {
      ok = false;
      break;
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// Byte offset of 16-byte chunk `ch` of row `row` in a 128-byte-row tile with
// the 128-byte swizzle (the layout TMA writes and UMMA reads).
__device__ __forceinline__ uint32_t sw128_off(int row, int ch) {
  return uint32_t(row) * 128u + (uint32_t(ch ^ (row & 7)) << 4);
}

// The low bytes of four int32 values, packed little-endian into one word.
__device__ __forceinline__ uint32_t low_bytes4(const uint32_t* v) {
  return __byte_perm(__byte_perm(v[0], v[1], 0x0040), __byte_perm(v[2], v[3], 0x0040), 0x5410);
}

// Four byte-wise additions modulo 256 in one word: the low seven bits of
// each byte add without reaching the next byte, the top bit is their carry
// XOR the two top bits.  Equals int8(x_b + y_b) for every byte b.
__device__ __forceinline__ uint32_t add_bytes4(uint32_t x, uint32_t y) {
  return ((x & 0x7F7F7F7Fu) + (y & 0x7F7F7F7Fu)) ^ ((x ^ y) & 0x80808080u);
}

// Per k-block of one CTA (256 rows of X, 128 columns of k):
//   producer  TMA the E_rmajor / E_kmajor tiles (signalled separately, they
//             serve both 128-row halves) and then the X tile into one of
//             three stages
//   MMA       D1_h = EL_h . E_rmajor^T for the two row halves h (one TMEM
//             buffer, 2 x 128 columns) as soon as the E tiles land;
//             D2_h += Xs_h . E_kmajor^T
//   epilogue  16 warps, one per (row half, TMEM lane quadrant, column
//             half), read their rows of D1 and pack the low bytes while X is in
//             flight, then add them into the X tile in place, four bytes per
//             instruction (the tile becomes the XpE tile in the same swizzled
//             operand layout), and store their 32 x 64 blocks with coalesced
//             16-byte stores; the stage is free once every warp has stored and the
//             MMA has read it
// noise_A's projection reads the original X: it is issued when X lands and
// the epilogue rewrites X only after it (x_free).  noise_B's projection reads
// XpE: it is issued once all epilogue warps have published the rewritten tile.
template <int R, bool kB>
__device__ __forceinline__ void noising_body(const NoisingArgs& a) {
  constexpr int kE1Bytes = NKB * R;
  constexpr int kE2Bytes = R * NKB;
  constexpr uint32_t kIdesc1 = idesc_i8(128, NKB);
  constexpr uint32_t kIdesc2 = idesc_i8(128, R);
  constexpr uint32_t kD2 = 256;  // TMEM column of D2_0; D2_1 follows at + R

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* el_buf = base;
  uint8_t* stages = base + kElBytes;
  NSmem& S = *reinterpret_cast<NSmem*>(base + kSmemPlan);
  volatile int* abort_flag = &S.abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb0 = blockIdx.y * a.kbps;
  const int nkb = min(a.kbps, a.nkb - kb0);
  const int r0 = blockIdx.x * a.nm;
  const uint32_t rank = a.use_cluster ? cluster_ctarank() : 0;
  bool waited_cluster = false;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&S.full_e[i], 1);
      mbar_init(&S.full_x[i], 1);
      mbar_init(&S.x_free[i], 1);
      mbar_init(&S.empty[i], 1 + kEpiWarps);  // MMA commit + every epilogue warp
      mbar_init(&S.xp_ready[i], kEpiWarps);
    }
    mbar_init(&S.el_full, 1);
    mbar_init(&S.d1_full, 1);
    mbar_init(&S.d1_empty, kEpiWarps);
    mbar_init(&S.d2_full, 1);
    mbar_init(&S.red_ready, kEpiWarps * (a.use_cluster ? a.ks : 1));
    mbar_init(&S.red_done, kEpiWarps * (a.use_cluster ? a.ks : 1));
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
  // Set-up above touches no global memory; it overlaps the previous kernel.
  griddep_wait();
  griddep_launch_dependents();
  // Peers are touched only in the projection tail: announce this CTA's
  // barriers now and wait for the peers' just before the first remote access.
  if (a.use_cluster) cluster_arrive();
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the k-blocks; one elected lane issues the loads.
    {
      const bool leader = elect_one();
      if (leader) {
        tma_prefetch(&a.tmX);
        tma_prefetch(&a.tmE1);
        tma_prefetch(&a.tmE2);
        mbar_arrive_expect_tx(&S.el_full, a.nm * R);
        tma_load_2d(&a.tmEL, &S.el_full, el_buf, 0, r0);
      }
      int i = 0;
      for (; i < nkb; ++i) {
        const int s = i % kStages;
        if (!mbar_wait_warp(&S.empty[s], ((i / kStages) & 1) ^ 1, abort_flag, a.sync, a.wait_budget)) break;
        uint8_t* st = stages + s * kStageSlot;
        const int k = (kb0 + i) * NKB;
        if (leader) {
          // E first: the noise tile is computed from it while X is in flight.
          mbar_arrive_expect_tx(&S.full_e[s], kE1Bytes + kE2Bytes);
          tma_load_2d(&a.tmE1, &S.full_e[s], st + kXBytes, 0, k);
          tma_load_2d(&a.tmE2, &S.full_e[s], st + kXBytes + 16384, k, 0);
          mbar_arrive_expect_tx(&S.full_x[s], a.nm * NKB);
          tma_load_2d(&a.tmX, &S.full_x[s], st, k, r0);
        }
      }
      for (int j = (i > kStages ? i - kStages : 0); j < i; ++j) {
        long long t0 = clock64();
        while (!(mbar_test(&S.full_e[j % kStages], (j / kStages) & 1) &&
                 mbar_test(&S.full_x[j % kStages], (j / kStages) & 1)) &&
               clock64() - t0 < 100000000LL) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the issue loop; one elected lane issues each MMA
    // and commit (the *_warp forms).
    {
      bool ok = mbar_wait_warp(&S.el_full, 0, abort_flag, a.sync, a.wait_budget);
      const uint32_t el = smem_u32(el_buf);
      // projection of k-block j: D2_h += Xs_h[j] . E_kmajor[j]^T
      auto mma2 = [&](int j) {
        const uint32_t st = smem_u32(stages + (j % kStages) * kStageSlot);
        const uint64_t bd = sdesc_kmajor<128>(st + kXBytes + 16384);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint64_t ad = sdesc_kmajor<128>(st + h * (kXBytes / 2));
#pragma unroll
          for (int ks = 0; ks < NKB / 32; ++ks)
            umma_i8_warp(tmem + kD2 + h * R, ad + 2 * ks, bd + 2 * ks, kIdesc2, (j | ks) != 0);
        }
      };
      // projection of k-block j, once its operand is in place: the original X
      // (noise_A; the epilogue rewrites it after x_free) or the XpE tile the
      // epilogue published (noise_B)
      auto proj = [&](int j) -> bool {
        const int s = j % kStages;
        uint64_t* ready = kB ? &S.xp_ready[s] : &S.full_x[s];
        if (!mbar_wait_warp(ready, (j / kStages) & 1, abort_flag, a.sync, a.wait_budget)) return false;
        tc_fence_after();
        mma2(j);
        if (!kB) umma_commit_warp(&S.x_free[s]);
        umma_commit_warp(&S.empty[s]);
        return true;
      };
      // D1 of k-block i needs only the E tiles.  noise_B's projection of
      // k-block i waits for the epilogue, so D1 runs one k-block ahead of it;
      // noise_A's follows its own D1 at once (the epilogue's rewrite of X
      // waits for it).
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % kStages;
        if (!(ok = mbar_wait_warp(&S.full_e[s], (i / kStages) & 1, abort_flag, a.sync, a.wait_budget))) break;
        if (i >= 1 && !(ok = mbar_wait_warp(&S.d1_empty, (i - 1) & 1, abort_flag, a.sync, a.wait_budget))) break;
        tc_fence_after();
        {
          const uint64_t bd = sdesc_kmajor<R>(smem_u32(stages + s * kStageSlot + kXBytes));
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t ad = sdesc_kmajor<R>(el + h * 128 * R);  // rows 128h..
#pragma unroll
            for (int ks = 0; ks < R / 32; ++ks)
              umma_i8_warp(tmem + 128 * h, ad + 2 * ks, bd + 2 * ks, kIdesc1, ks != 0);
          }
          umma_commit_warp(&S.d1_full);
        }
        if (!kB) ok = proj(i);
        else if (i >= 1) ok = proj(i - 1);
      }
      if (ok && kB && nkb >= 1) ok = proj(nkb - 1);
      umma_commit_warp(&S.d2_full);
      umma_commit_warp(&S.drain);
      long long t0 = clock64();
      while (!mbar_test(&S.drain, 0) && clock64() - t0 < 100000000LL) {
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;
    const int q = warp & 3;               // TMEM lane quadrant this warp may read
    const int h = (e >> 2) & 1;           // row half (MMA accumulator) of this warp
    const int c2 = e >> 3;                // 64-column half of the k-block
    const int row = 128 * h + 32 * q + lane;  // row of the CTA tile this thread owns
    const uint32_t trow = tmem + (uint32_t(32 * q) << 16);
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      const int s = i % kStages;
      if (!(ok = mbar_wait_warp(&S.d1_full, i & 1, abort_flag, a.sync, a.wait_budget))) break;
      tc_fence_after();
      // The noise bytes of this thread's row, packed while X is in flight.
      uint32_t nz[16];
      {
        uint32_t v[2][32];
        tmem_ld32(trow + 128 * h + 64 * c2, v[0]);
        tmem_ld32(trow + 128 * h + 64 * c2 + 32, v[1]);
        tmem_wait_ld_into(v[0]);
        tmem_wait_ld_into(v[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.d1_empty);
#pragma unroll
        for (int w = 0; w < 16; ++w) nz[w] = low_bytes4(v[w >> 3] + 4 * (w & 7));
      }
      // X landed (and, for noise_A, the projection has read it).
      if (!(ok = mbar_wait_warp(&S.full_x[s], (i / kStages) & 1, abort_flag, a.sync, a.wait_budget))) break;
      if (!kB && !(ok = mbar_wait_warp(&S.x_free[s], (i / kStages) & 1, abort_flag, a.sync, a.wait_budget))) break;
      uint8_t* xt = stages + s * kStageSlot;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4* px = reinterpret_cast<uint4*>(xt + sw128_off(row, 4 * c2 + j));
        const uint4 xv = *px;
        *px = make_uint4(add_bytes4(xv.x, nz[4 * j]), add_bytes4(xv.y, nz[4 * j + 1]),
                         add_bytes4(xv.z, nz[4 * j + 2]), add_bytes4(xv.w, nz[4 * j + 3]));
      }
      if (kB) fence_proxy_async_smem();  // the projection MMA reads the XpE tile
      __syncwarp();
      if (kB && lane == 0) mbar_arrive(&S.xp_ready[s]);
      // This warp's 32 x 64 block of XpE to global memory, 64 contiguous
      // bytes of a row per 4 lanes (the thread-per-row layout above would
      // scatter the stores).  The two rows of an 8-lane shared-memory
      // wavefront are 4 apart, so their swizzled chunks use all 8 bank groups.
      {
        const int ch = 4 * c2 + (lane & 3);
        const int sub = lane >> 2;
        const int64_t kc = int64_t(kb0 + i) * NKB + 16 * ch;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int rr = 128 * h + 32 * q + 8 * j + (sub >> 1) + 4 * (sub & 1);
          const uint4 val = *reinterpret_cast<const uint4*>(xt + sw128_off(rr, ch));
          const int64_t g = int64_t(r0) + rr;
          if (rr < a.nm && g < a.rows && kc < a.K) *reinterpret_cast<uint4*>(a.XpE + g * a.K + kc) = val;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[s]);
    }
    // ---- projection: D2 (256 x R int32) -> proj
    // Each CTA stages its partial in the (now idle) operand ring, row-major
    // with the 16-byte chunks of a row XOR-swizzled by the row so that the
    // thread-per-row writes are conflict-free.  Then every rank of the
    // cluster (one rank without a K split) sums a contiguous slice of the
    // rows over all ranks' partials, one row per warp with coalesced reads,
    // and writes fp16 (or adds into int32) with coalesced stores.
    constexpr int kChunks = R / 4;            // 16-byte chunks per row
    constexpr int kRowsPerIter = 32 / kChunks;  // rows a warp covers per pass
    int32_t* red = reinterpret_cast<int32_t*>(stages);
    const int nr = a.use_cluster ? a.ks : 1;
    ok = ok && mbar_wait_warp(&S.d2_full, 0, abort_flag, a.sync, a.wait_budget);
    // The partial overwrites the ring: every epilogue warp is done with it.
    ok = named_barrier_and(1, 32 * kEpiWarps, ok);
    if (a.use_cluster) {
      cluster_wait();  // every peer's barriers are initialized
      waited_cluster = true;
    }
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c = c2 * (R / 2); c < (c2 + 1) * (R / 2); c += 32) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(trow + kD2 + h * R + c, v);
        tmem_wait_ld_into(v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int ch = c / 4 + j;
          *reinterpret_cast<int4*>(red + row * R + 4 * (ch ^ (row & (kChunks - 1)))) =
              make_int4(int(v[4 * j]), int(v[4 * j + 1]), int(v[4 * j + 2]), int(v[4 * j + 3]));
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (a.use_cluster) {
          for (int r = 0; r < nr; ++r) mbar_arrive_remote(mapa(&S.red_ready, uint32_t(r)));
        } else {
          mbar_arrive(&S.red_ready);
        }
      }
      ok = a.use_cluster ? wait_cluster_bounded(&S.red_ready, 0, a.wait_budget)
                         : mbar_wait_warp(&S.red_ready, 0, abort_flag, a.sync, a.wait_budget);
    }
    if (ok) {
      const int per = (a.nm + nr - 1) / nr;
      const int lo = int(rank) * per, hi = min(a.nm, lo + per);
      const int sub = lane / kChunks, cl = lane % kChunks;
      constexpr int kStep = kEpiWarps * kRowsPerIter;  // rows between a thread's rows
      // Two rows per pass with every rank's partial of both in flight (one
      // round trip per pass rather than one per rank).
#pragma unroll 1
      for (int r0w = lo + e * kRowsPerIter + sub; r0w < hi; r0w += 2 * kStep) {
        int4 pv[2][8];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int rr = r0w + j * kStep;
          const int32_t* src = red + rr * R + 4 * (cl ^ (rr & (kChunks - 1)));
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            pv[j][r] = make_int4(0, 0, 0, 0);
            if (rr < hi && r < nr)
              pv[j][r] = a.use_cluster ? ld_cluster_v4(mapa(src, uint32_t(r)))
                                       : *reinterpret_cast<const int4*>(src);
          }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int rr = r0w + j * kStep;
          int4 s = pv[j][0];
#pragma unroll
          for (int r = 1; r < 8; ++r) {
            s.x += pv[j][r].x; s.y += pv[j][r].y; s.z += pv[j][r].z; s.w += pv[j][r].w;
          }
          const int64_t g = int64_t(r0) + rr;
          if (rr < hi && g < a.rows) {
            if (a.proj_fp16) {
              const __half2 lo2 = __floats2half2_rn(float(s.x) * a.scale, float(s.y) * a.scale);
              const __half2 hi2 = __floats2half2_rn(float(s.z) * a.scale, float(s.w) * a.scale);
              uint2 o;
              o.x = *reinterpret_cast<const uint32_t*>(&lo2);
              o.y = *reinterpret_cast<const uint32_t*>(&hi2);
              *reinterpret_cast<uint2*>(static_cast<__half*>(a.proj) + g * R + 4 * cl) = o;
            } else {
              int* o = static_cast<int*>(a.proj) + g * R + 4 * cl;
              atomicAdd(o, s.x); atomicAdd(o + 1, s.y); atomicAdd(o + 2, s.z); atomicAdd(o + 3, s.w);
            }
          }
        }
      }
      if (a.use_cluster) {
        // stay resident until every rank has read this CTA's partial
        __syncwarp();
        if (lane == 0)
          for (int r = 0; r < nr; ++r) mbar_arrive_remote(mapa(&S.red_done, uint32_t(r)));
        if (!wait_cluster_bounded(&S.red_done, 0, a.wait_budget)) ok = false;
      }
    }
  }

  // Warps that did not wait on the cluster barrier above do it here: no CTA
  // leaves before all of the cluster has arrived.
  if (a.use_cluster && !waited_cluster) cluster_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

template <int R, bool kB>
__global__ void __launch_bounds__(kThreads, 1) noising_kernel(const __grid_constant__ NoisingArgs a) {
  noising_body<R, kB>(a);
}

// noise_A and noise_B of one mined GEMM in a single launch (blockIdx.z picks
// the operand): they are independent, and one launch pays the launch, the
// pipeline fill and the cluster reduction once for both.  Clusters run along
// y, so the CTAs of a row block beyond one operand's rows leave together.
template <int R>
__global__ void __launch_bounds__(kThreads, 1)
    noising_pair_kernel(const __grid_constant__ NoisingArgs a, const __grid_constant__ NoisingArgs b) {
  if (blockIdx.z == 0) {
    if (int(blockIdx.x) * a.nm < a.rows) noising_body<R, false>(a);
  } else {
    if (int(blockIdx.x) * b.nm < b.rows) noising_body<R, true>(b);
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
  cudaLaunchAttribute attr[2];
  unsigned nattr = 0;
  attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait
  attr[nattr++].val.programmaticStreamSerializationAllowed = 1;
  if (a.use_cluster) {
    attr[nattr].id = cudaLaunchAttributeClusterDimension;
    attr[nattr].val.clusterDim.x = 1;
    attr[nattr].val.clusterDim.y = unsigned(a.ks);
    attr[nattr++].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  cudaLaunchKernelEx(&cfg, kern, a);
  return launch_status();
}

// How many clusters of `ks` noising CTAs the device holds at once (-1 if the
// query fails).  Every instantiation has the same block size and shared
// memory, so one kernel stands for all of them.  Cached per device.
int max_active_clusters(int device, int ks) {
  static int cache[64][9];
  if (device < 0 || device >= 64 || ks < 1 || ks > 8) return -1;
  if (cache[device][ks] != 0) return cache[device][ks] - 2;
  auto kern = noising_kernel<128, false>;
  const int smem = kSmemPlan + int(sizeof(NSmem)) + 1024;
  int n = -1;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, unsigned(ks), 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = size_t(smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = unsigned(ks);
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = -1;
  }
  (void)cudaGetLastError();
  cache[device][ks] = n + 2;
  return n;
}

// Rows of X per CTA: the tensor maps of X and EL load boxes nm rows high.
int set_rows_per_block(NoisingArgs& a, const pb2_noising_params& p, int nm) {
  const CUtensorMapSwizzle rswz = p.r == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  int st;
  if ((st = make_tmap_2d(&a.tmX, p.X, U8, 1, p.k, p.rows, NKB, nm, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (st = make_tmap_2d(&a.tmEL, p.EL, U8, 1, int(p.r), p.rows, int(p.r), nm, rswz)))
    return st;
  a.nm = nm;
  return PB2_OK;
}

// The smallest row block (a multiple of 8 in [128, NM]) whose blocks, for
// operands of rows_a and rows_b rows, still run as one wave of ks-CTA
// clusters: more of the SMs stream X, each with less of it (at 8192 rows per
// operand and ks = 2: 224-row blocks, 148 CTAs, against 128 CTAs of 256).
int rows_per_block(int device, int64_t rows_a, int64_t rows_b, int ks) {
  const int sms = std::max(1, sm_count(device));
  int cap = sms / std::max(1, ks);
  if (ks > 1) {
    const int fit = max_active_clusters(device, ks);
    if (fit >= 0) cap = std::min(cap, fit);
  }
  for (int nm = 128; nm < NM; nm += 8)
    if ((rows_a + nm - 1) / nm + (rows_b + nm - 1) / nm <= cap) return nm;
  return NM;
}

// Validates one operand's parameters and fills its arguments except the K
// split (kbps, ks, use_cluster); the row block is NM until a caller sets it.
int prepare_noising(const pb2_noising_params& p, bool b_side, NoisingArgs* out) {
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
  NoisingArgs& a = *out;
  std::memset(&a, 0, sizeof(a));
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if ((st = set_rows_per_block(a, p, NM)) ||
      (st = make_tmap_2d(&a.tmE1, p.E_rmajor, U8, 1, r, p.k, r, NKB, rswz)) ||
      (st = make_tmap_2d(&a.tmE2, p.E_kmajor, U8, 1, p.k, r, NKB, r, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  a.rows = int(p.rows);
  a.K = int(p.k);
  a.nkb = int((p.k + NKB - 1) / NKB);
  a.proj_fp16 = p.proj_is_fp16;
  a.scale = b_side ? (1.0f / 4096.0f) : (1.0f / 16384.0f);
  a.XpE = static_cast<int8_t*>(p.XpE);
  a.proj = p.proj;
  a.sync = static_cast<SignalSync*>(p.host_signal_sync);
  // Always the default budget, never the process-wide one: a CTA of a
  // K-split cluster leaves only after its peers have read its partial (the
  // red_done handshake), and a budget short enough to cut that wait would
  // let peers read the shared memory of a CTA that has left.
  a.wait_budget = kWaitBudgetCycles;
  return PB2_OK;
}

// K split of a half-precision projection: over a cluster (<= 8 CTAs) so
// that one wave covers the GPU, the widest split whose clusters (one per row
// block) are all resident at once.
int fp16_split(int device, int row_blocks, int nkb) {
  const int sms = std::max(1, sm_count(device));
  int ks = std::max(1, std::min({8, nkb, sms / row_blocks}));
  while (ks > 1) {
    const int fit = max_active_clusters(device, ks);
    if (fit < 0 || fit >= row_blocks) break;
    --ks;
  }
  return ks;
}

void set_split(NoisingArgs& a, int ks) {
  a.kbps = (a.nkb + ks - 1) / ks;
  a.ks = (a.nkb + a.kbps - 1) / a.kbps;
  a.use_cluster = a.proj_fp16 && a.ks > 1;
}

int run_noising(const pb2_noising_params& p, bool b_side, cudaStream_t stream) {
  NoisingArgs a;
  int st = prepare_noising(p, b_side, &a);
  if (st) return st;
  int row_blocks = int((p.rows + NM - 1) / NM);
  const int sms = std::max(1, sm_count(p.device));
  int ks;
  if (p.proj_is_fp16) {
    ks = fp16_split(p.device, row_blocks, a.nkb);
    if ((st = set_rows_per_block(a, p, rows_per_block(p.device, p.rows, 0, ks)))) return st;
    row_blocks = int((p.rows + a.nm - 1) / a.nm);
  } else if (p.k_blocks_per_split > 0) {
    ks = (a.nkb + p.k_blocks_per_split - 1) / p.k_blocks_per_split;
  } else if (p.k_blocks_per_split == 0) {
    ks = 1;
  } else {
    ks = std::max(1, std::min(a.nkb, (sms + row_blocks - 1) / row_blocks));
  }
  set_split(a, ks);
  if (p.r == 128) return b_side ? launch_noising<128, true>(a, row_blocks, stream)
                                : launch_noising<128, false>(a, row_blocks, stream);
  return b_side ? launch_noising<64, true>(a, row_blocks, stream)
                : launch_noising<64, false>(a, row_blocks, stream);
}

template <int R>
int launch_noising_pair(const NoisingArgs& a, const NoisingArgs& b, int row_blocks, cudaStream_t s) {
  auto kern = noising_pair_kernel<R>;
  const int smem = kSmemPlan + int(sizeof(NSmem)) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(row_blocks), unsigned(a.ks), 2);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned nattr = 0;
  attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait
  attr[nattr++].val.programmaticStreamSerializationAllowed = 1;
  if (a.use_cluster) {
    attr[nattr].id = cudaLaunchAttributeClusterDimension;
    attr[nattr].val.clusterDim.x = 1;
    attr[nattr].val.clusterDim.y = unsigned(a.ks);
    attr[nattr++].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  cudaLaunchKernelEx(&cfg, kern, a, b);
  return launch_status();
}

}  // namespace

// noise_A then noise_B, as one launch when both projections are half
// precision with the same rank and K (the mined GEMM's usual case), else as
// two.
int run_noising_both(const pb2_noising_params& pa, const pb2_noising_params& pb, cudaStream_t stream) {
  if (!(pa.proj_is_fp16 && pb.proj_is_fp16 && pa.r == pb.r && pa.k == pb.k && pa.device == pb.device)) {
    int st = run_noising(pa, false, stream);
    return st ? st : run_noising(pb, true, stream);
  }
  NoisingArgs a, b;
  int st = prepare_noising(pa, false, &a);
  if (st || (st = prepare_noising(pb, true, &b))) return st;
  const int ks = fp16_split(pa.device, int((pa.rows + NM - 1) / NM + (pb.rows + NM - 1) / NM), a.nkb);
  const int nm = rows_per_block(pa.device, pa.rows, pb.rows, ks);
  if ((st = set_rows_per_block(a, pa, nm)) || (st = set_rows_per_block(b, pb, nm))) return st;
  set_split(a, ks);
  set_split(b, ks);
  const int rb = int(std::max((pa.rows + nm - 1) / nm, (pb.rows + nm - 1) / nm));
  return pa.r == 128 ? launch_noising_pair<128>(a, b, rb, stream) : launch_noising_pair<64>(a, b, rb, stream);
}

namespace {

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
  pb2::NvtxRange nvtx_range("pb2_noise_A");
  if (!p) return PB2_ERR_INVALID_ARGUMENT;
  return pb2::run_noising(*p, false, static_cast<cudaStream_t>(stream));
}

extern "C" int pb2_noise_B(const pb2_noising_params* p, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_noise_B");
  if (!p) return PB2_ERR_INVALID_ARGUMENT;
  return pb2::run_noising(*p, true, static_cast<cudaStream_t>(stream));
}

extern "C" int pb2_noise_AB(const pb2_noising_params* a, const pb2_noising_params* b, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_noise_AB");
  if (!a || !b) return PB2_ERR_INVALID_ARGUMENT;
  return pb2::run_noising_both(*a, *b, static_cast<cudaStream_t>(stream));
}

extern "C" int pb2_denoise_converter(const pb2_denoise_converter_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_denoise_converter");
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
