// noisy_gemm.cu -- the mined GEMM on sm_100a tensor cores.
//
// A cluster of two CTAs (one per SM) computes 256 x 256 output tiles with
// 2-SM MMAs (tcgen05.mma.cta_group::2, int8 x int8 -> int32): each CTA loads
// 128 rows of ApEA and half of the 256 BpEB rows per K stage, so an SM streams
// 32 KB per 128 bytes of K and the leader CTA issues one M=256, N=256 MMA per
// 32 bytes of K.  Each CTA's tensor memory (512 columns) holds its 128 x 256
// half of two independent tiles ("slots"); the leader issues the slots'
// R-chunks of K in strict alternation, so while the tensor core runs one
// slot's chunk the epilogue reads the other slot's running accumulator for
// the transcript -- the MMA does not wait for a fold.
//
// Transcript (protocol: zk-pow/src/ffi/mine.rs:86-107; GPU twin
// pearl-gemm/csrc/gemm/pow_utils.hpp:129-200, collective_mainloop.hpp:270-317):
// after each R-chunk a slot's accumulator is read by 16 fold warps (4 per
// TMEM lane quadrant, 64 columns each, 32x32b loads) and XOR-folded onto the
// protocol's 2 x 64 hash tiles (rows {r, r+8} x cols {c + 8j, c + 8j + 1});
// one thread per hash tile rotate-xors the folded word into word (chunk % 16)
// of the tile's register transcript.  Fold and rotate-xor are GF(2)-linear,
// so the per-strip partial folds simply XOR together.  Reading 128 KB of TMEM
// per chunk at full MMA rate needs ~256 B/cycle per SM; 16 warps of 32x32b
// loads deliver ~470.

// Epilogue (collective_epilogue.hpp:361-599 semantics): the final int32
// accumulator is rewritten in TMEM as f32 * 2^-12, f16 2-SM MMAs add the
// low-rank denoise terms EAL_fp16 . EARxBpEB_fp16^T + AxEBL_fp16 . EBR_fp16^T,
// and C = bf16(D * 2^12 * A_scales[m] * B_scales[n]) is stored.  Two hash
// warps per CTA combine the partial transcripts, hash each tile with keyed
// BLAKE3 (pow_utils.hpp:205-234) and compare with the uint256 target; hits
// are published without any spin lock (the first hit claims the pinned host
// header with one atomicCAS).
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <type_traits>

#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int BMC = 128;     // rows per CTA (half of the pair tile)
constexpr int BM = 2 * BMC;  // rows per pair tile
constexpr int BN = 256;
constexpr int kTileK = 128;  // the reference's tile_size_k (K must be a multiple)
constexpr int kFoldWarps = 16;
constexpr int kHashWarps = 2;
constexpr int kThreads = 32 * (2 + kFoldWarps + kHashWarps);  // TMA, MMA, fold, hash
// Operand ring bytes: shared memory (227 KB per CTA) also holds the C boxes
// and, with the transcript, 64 KB of transcript buffers.
constexpr int stage_budget(bool reduce) { return reduce ? 128 * 1024 : 160 * 1024; }
constexpr int kMaxStages = 8;
constexpr int kXbufBytes = 4 * 16 * 256 * 4;  // transcripts of 256 hash tiles, 2 slots x 2 tiles in flight
constexpr int kCBoxBytes = 32 * 32 * 2;         // one fold warp's C box: 32 rows x 32 bf16 columns
constexpr int kCStageBytes = kFoldWarps * kCBoxBytes;
constexpr int kTmemCols = 512;
constexpr uint16_t kPairMask = 0x3;

// What one launch shares: the B-side operands (the rows of every problem's
// B), the shapes, the schedule and the hash inputs.
struct MainArgs {
  CUtensorMap tmB;           // BpEB (n_rows,k) int8
  CUtensorMap tmDB0, tmDB1;  // EARxBpEB_fp16, EBR_fp16 (n_rows,r)
  int N, K, R;               // N: columns of C (rows of B per problem)
  int tiles_n, num_tiles, group;
  int tpr;  // tiles a CTA pair runs per round: 2 (two TMEM slots in alternation) or 1
  int scale_per_tensor;  // sA[0] and sB[0] scale every row and column (FP8 operands)
  // Plain GEMM only: K split into `ksplit` equal ranges, one work item per
  // (tile, range); each item writes its exact int32 partial to ws[range] and
  // a reduction kernel sums the ranges and scales (1: no split).
  int ksplit;
  int32_t* ws;  // (ksplit, m, N) int32
  CUtensorMap tmW;  // ws as (N, m, ksplit) int32, 16 x 32 boxes, 64-byte swizzle (split-K only)
  // Grouped launch with a row map (ExpertEntry::c_rows): C's destination
  // (c_dst_rows rows of N bf16).
  uint16_t* c_dst;
  long long c_dst_rows;
  SignalSync* sync;  // where a timed-out wait records its error
  const uint32_t* target;
  const uint32_t* key;
  unsigned long long* counter;
  long long wait_budget;  // SM cycles a device-side wait may spin (pb2_set_wait_budget_cycles)
  uint32_t wait_hint_ns;  // suspend hint of those waits, derived from the budget (suspend_hint_ns)
};

// One GEMM of the launch: the whole problem of pb2_noisy_gemm, or one expert
// of pb2_noisy_gemm_grouped (its rows of A and C, its n rows of B, its own
// hit signalling).  The A-side tensor maps cover exactly the problem's rows,
// so loads past its last row read the fill value and stores past it are
// dropped, as in a launch of its own.
struct ExpertEntry {
  CUtensorMap tmA;           // ApEA rows (m,k) int8, boxes of 128 rows
  CUtensorMap tmDA0, tmDA1;  // EAL_fp16, AxEBL_fp16 rows (m,r)
  CUtensorMap tmC;           // C rows (m,N) bf16, 32 x 32 boxes, 64-byte swizzle
  int m;                     // rows
  int tiles_m;               // 256-row tiles
  int tile_begin;            // its first tile in the launch's tile order
  int b_row0;                // its first row of the B-side operands
  const float* sA;           // its A_scales
  const float* sB;           // its B_scales (N)
  SignalSync* sync;
  SignalHeader* header;
  uint32_t* hits;
  long long hit_cap;
  uint32_t* transcripts;
  uint32_t* digests;
  // Optional: row r of this problem's C goes to row c_rows[r] of a.c_dst
  // (the MoE slot-order write-back fused into the epilogue); null: tmC.
  const int32_t* c_rows;
};
constexpr int kMaxExperts = 16;  // experts of one grouped launch (kernel parameter space)
template <int kE>
struct ExpertTable {
  int count;
  ExpertEntry ex[kE];
};

struct TileRef {
  int e, tm, tn;
  int ks;  // K range of a split-K work item (0 without a split)
};

struct Smem {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];  // stage consumed: also "this transcript chunk is final"
  uint64_t acc_full[2];        // the slot's accumulator is final (denoise / store events)
  uint64_t acc_empty[2];
  uint64_t xready[4];  // transcript buffer 2 * slot + (round & 1) is complete
  uint64_t xfree[4];   // ... has been hashed and cleared
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// Tile t of the launch: its problem e and its (tm, tn) there.  Problems
// follow one another in tile order; within one, a raster of `group` row
// tiles walks all column tiles before the next group (L2 reuse of B).
template <int kE>
__device__ __forceinline__ TileRef tile_of(const MainArgs& a, const ExpertTable<kE>& x, int t) {
  int e = 0;
  if constexpr (kE > 1) {
    while (e + 1 < x.count && t >= x.ex[e + 1].tile_begin) ++e;
  }
  const ExpertEntry& E = x.ex[e];
  const int lt = t - E.tile_begin;
  const int group = min(a.group, E.tiles_m);
  const int gsize = group * a.tiles_n;
  const int g = lt / gsize;
  const int first_m = g * group;
  const int gm = min(group, E.tiles_m - first_m);
  const int within = lt - g * gsize;
  return TileRef{e, first_m + within % gm, within / gm, 0};
}

// Work item t of the launch: tile t, or with a K split tile t / ksplit and
// K range t % ksplit (the ranges of one tile follow one another).
template <int kE>
__device__ __forceinline__ TileRef item_of(const MainArgs& a, const ExpertTable<kE>& x, int t) {
  if (a.ksplit <= 1) return tile_of(a, x, t);
  const int tile = t / a.ksplit;
  TileRef r = tile_of(a, x, tile);
  r.ks = t - tile * a.ksplit;
  return r;
}

// Per-slot phase bits packed in one word (bit s = parity of slot s).
__device__ __forceinline__ uint32_t bit(uint32_t w, int s) { return (w >> s) & 1u; }

__device__ __forceinline__ uint32_t pack_bf16(float x, float y) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One fold warp's 32 x 32 block of C (lane = row, `w` = the row's 32 bf16
// values as 16 packed pairs): write the block into the warp's shared-memory
// box and hand it to a TMA store, which writes whole lines and clips rows >= M
// and columns >= N.  Writing C straight from registers would scatter every
// store instruction over 32 rows, and the fold warps would spend thousands of
// cycles in the store unit while the MMA issuer waits for their next release.
__device__ __forceinline__ void store_c_packed(const CUtensorMap* tmC, uint8_t* box, const uint32_t* w,
                                               int row0, int col0, int lane) {
  if (lane == 0) bulk_wait_read_all();  // the box's previous store has read it
  __syncwarp();
  // 64-byte swizzle (the tensor map's): 16-byte chunk k of row r sits at
  // chunk k ^ ((r >> 1) & 3), which also spreads a store instruction's 32
  // lanes over all banks.
  uint8_t* rowp = box + lane * 64;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    *reinterpret_cast<uint4*>(rowp + ((k ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmC, box, col0, row0);
    bulk_commit_group();
  }
}

// Hit publication.  Rows are reported in the reference's 128-row tile
// convention (tileCoord[0] = 128-row block, thread rows < 128), so
// extract_indices() gives the same A rows as for the reference kernel.
__device__ void publish_hit(const MainArgs& a, const ExpertEntry& E, int tm128, int tn, int row_in_tile,
                            int cls, const uint32_t* digest) {
  const uint32_t row_off = uint32_t(tm128 * BMC + row_in_tile);
  const uint32_t col_off = uint32_t(tn * BN + 2 * cls);
  const unsigned slot = atomicAdd(&E.sync->hit_count, 1u);
  if (E.hits && (long long)slot < E.hit_cap) {
    uint32_t* h = E.hits + size_t(slot) * PB2_HIT_WORDS;
    h[0] = row_off;
    h[1] = col_off;
    h[2] = uint32_t(tm128);
    h[3] = uint32_t(tn);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[4 + i] = digest[i];
  }
  if (E.header && atomicCAS(&E.sync->global_lock, 0, 1) == 0) {
    SignalHeader* H = E.header;
    H->gridDim[0] = gridDim.x; H->gridDim[1] = gridDim.y; H->gridDim[2] = gridDim.z;
    H->blockDim[0] = blockDim.x; H->blockDim[1] = blockDim.y; H->blockDim[2] = blockDim.z;
    H->blockIdx[0] = blockIdx.x; H->blockIdx[1] = blockIdx.y; H->blockIdx[2] = blockIdx.z;
    H->tileCoord[0] = uint32_t(tm128); H->tileCoord[1] = uint32_t(tn); H->tileCoord[2] = 0;
    H->threadIdx[0] = threadIdx.x; H->threadIdx[1] = 0; H->threadIdx[2] = 0;
    H->num_registers_per_thread = 128;
    // Element j of the hash tile, in the reference's per-thread fragment
    // order: (row r, col c), (r, c+1), (r+8, c), (r+8, c+1), then c += 8.
    for (int j = 0; j < 128; ++j) {
      H->thread_rows[j] = uint8_t(row_in_tile + 8 * ((j >> 1) & 1));
      H->thread_cols[j] = uint8_t(2 * cls + (j & 1) + 8 * (j >> 2));
    }
    H->mma_size[0] = E.m; H->mma_size[1] = a.N; H->mma_size[2] = a.K;
    H->mma_tile_size[0] = BMC; H->mma_tile_size[1] = BN; H->mma_tile_size[2] = kTileK;
    for (int i = 0; i < 8; ++i) H->target[i] = a.target[i];
    __threadfence_system();
    H->status = 1;
    __threadfence_system();
    atomicExch(&E.sync->status, 1);
  }
}

// kSPU = operand stages per unit (1, or 2 for R = 256): a compile-time unit
// keeps the per-unit bookkeeping of the producer, issuer and fold warps free
// of runtime loops and divisions (measured: several hundred cycles per unit
// on the issuer otherwise).
//
// kTN = tile width: 256, or 128 for the plain GEMM of small problems (fewer
// than two 256-wide tiles per SM pair: a decode batch), where narrower tiles
// put more of the 148 SMs to work; the transcript and denoise variants
// always use 256 (the hash-tile column period).
//
// kE = problems per launch: 1, or up to kMaxExperts (the grouped MoE GEMM:
// every expert's tiles in one persistent launch, x.ex[e] per expert).
//
// kKind = operand type: 0 = int8 (kind::i8, int32 accumulators), 1 = FP8
// E4M3, 2 = FP8 E5M2 (kind::f8f6f4, f32 accumulators whose bit patterns the
// transcript folds; no noising or denoise terms).
template <int BK, int kSPU, bool kReduce, bool kDenoise, bool kDebug, int kTN, int kE, int kKind = 0>
__global__ void __launch_bounds__(kThreads, 1)
    noisy_gemm_kernel(const __grid_constant__ MainArgs a, const __grid_constant__ ExpertTable<kE> x) {
  static_assert(kKind == 0 || !kDenoise, "FP8 operands carry no denoise terms");
  static_assert(kTN == BN || (kTN == BN / 2 && !kReduce && !kDenoise), "narrow tiles: plain GEMM only");
  constexpr int kAStage = BMC * BK;        // this CTA's 128 rows of A
  constexpr int kBStage = (kTN / 2) * BK;  // this CTA's half of the tile's rows of B
  constexpr int kStageBytes = kAStage + kBStage;
  constexpr int kStageBudget = stage_budget(kReduce);
  constexpr int kStages =
      (kStageBudget / kStageBytes) < kMaxStages ? (kStageBudget / kStageBytes) : kMaxStages;
  // Split-K partials can be staged in the idle operand ring: 8 KB per fold warp.
  constexpr bool kRingStagesPartials = kStages * kStageBytes >= kFoldWarps * 8192;
  static_assert(kStageBudget + (kReduce ? kXbufBytes : 0) + kCStageBytes + 1024 + 256 <= 232448,
                "shared memory plan exceeds 227 KB");
  constexpr uint32_t kIdescI8 =
      kKind == 0 ? idesc_i8(BM, kTN) : idesc_f8(BM, kTN, uint32_t(kKind - 1), uint32_t(kKind - 1));
  constexpr uint32_t kIdescF16 = idesc_f16(BM, BN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_mem = base;
  uint32_t* xbuf = reinterpret_cast<uint32_t*>(base + kStageBudget);
  uint8_t* cstage = base + kStageBudget + (kReduce ? kXbufBytes : 0);
  Smem& S = *reinterpret_cast<Smem*>(cstage + kCStageBytes);
  volatile int* abort_flag = &S.abort_flag;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();  // 0 = leader (issues the MMAs), 1 = peer
  // A unit is one R-chunk of K (the transcript period) of one tile; without
  // transcript and denoise the chunk length only sets the interleaving.
  constexpr int unit_k = kSPU * BK;  // = R with transcript or denoise (host-checked)
  constexpr int stages_per_unit = kSPU;
  const int ksplit = a.ksplit > 1 ? a.ksplit : 1;
  const int nmain = a.K / unit_k / ksplit;  // units of one work item
  constexpr int nden = kDenoise ? 4 : 0;  // 2 products x 2R bytes of fp16 K = 4 units of R bytes
  const int units = nmain + nden;
  constexpr int den_stages_per_product = 2 * kSPU;
  // The producer asks L2 for the next round's first K stages when it reaches
  // main unit pf_unit of the current round (a few units before the tile end).
  constexpr int kPrefetchLead = 8;
  const int pf_unit = nmain > kPrefetchLead ? nmain - kPrefetchLead : 0;
  const int pf_stages = min(4, nmain * kSPU);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.acc_full[i], 1);
      mbar_init(&S.acc_empty[i], 2 * kFoldWarps);  // both CTAs' fold warps release a slot
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&S.xready[i], kFoldWarps);
      mbar_init(&S.xfree[i], kHashWarps);
    }
    mbar_init(&S.drain, 1);
    S.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&a.tmB);
    if (kDenoise) {
      tma_prefetch(&a.tmDB0);
      tma_prefetch(&a.tmDB1);
    }
    if constexpr (kE == 1) {
      tma_prefetch(&x.ex[0].tmA);
      tma_prefetch(&x.ex[0].tmC);
      if (kDenoise) {
        tma_prefetch(&x.ex[0].tmDA0);
        tma_prefetch(&x.ex[0].tmDA1);
      }
    }
  }
  if (warp == 1) {
    tmem_alloc_2sm(&S.tmem_base, kTmemCols);
    tmem_relinquish_2sm();
  }
  if (kReduce) {
    // Transcripts start at zero (the hash step clears them again afterwards).
    for (int i = threadIdx.x; i < kXbufBytes / 4; i += kThreads) xbuf[i] = 0u;
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or 2-SM load
  tc_fence_after();
  // Plain GEMM: the weights (B) are not produced by the kernel this launch
  // depends on, so the producer asks L2 for the B boxes of its first ring's
  // worth of stages before waiting for that kernel (an L2 prefetch is
  // coherent with whatever that kernel writes).  The first operand stage then
  // waits for the activations in L2, not for a weight round trip to HBM
  // (measured ~1.9 us after the wait in a decode chain without it).
  if constexpr (!kReduce && !kDenoise) {
    if (warp == 0 && elect_one()) {
      const int t0 = a.tpr * int(blockIdx.x >> 1);
      const int item_stages = a.K / BK / (a.ksplit > 1 ? a.ksplit : 1);
      int budget = kStages;
      for (int s = 0; s < a.tpr && t0 + s < a.num_tiles && budget > 0; ++s) {
        const TileRef r = item_of(a, x, t0 + s);
        const int n0 = x.ex[r.e].b_row0 + r.tn * kTN + int(rank) * (kTN / 2);
        const int n = min(item_stages, budget);
        for (int st = 0; st < n; ++st) tma_prefetch_l2_2d(&a.tmB, (r.ks * item_stages + st) * BK, n0);
        budget -= n;
      }
    }
  }
  // Set-up above touches no global memory but that L2 prefetch; it overlaps
  // the previous kernel.
  griddep_wait();
  griddep_launch_dependents();
  const uint32_t tmem = S.tmem_base;

  // Pair tiles are processed in rounds: round r holds tiles t0 = first + r *
  // stride (slot 0) and t0 + 1 (slot 1, when it exists and a.tpr == 2);
  // within a round the units alternate slot 0, slot 1.  Every role walks
  // this order.
  const int first = a.tpr * int(blockIdx.x >> 1);
  const int stride = a.tpr * int(gridDim.x >> 1);
  using I0 = std::integral_constant<int, 0>;
  using I1 = std::integral_constant<int, 1>;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the stage sequence; one elected lane issues the
    // arrivals and TMA loads.
    {
      const bool leader = elect_one();
      uint32_t it = 0;
      bool ok = true;
      for (int t0 = first; t0 < a.num_tiles && ok; t0 += stride) {
        const bool two = a.tpr == 2 && t0 + 1 < a.num_tiles;
        const TileRef r0 = item_of(a, x, t0);
        const TileRef r1 = two ? item_of(a, x, t0 + 1) : r0;
        const ExpertEntry& Ea = x.ex[r0.e];
        const ExpertEntry& Eb = x.ex[r1.e];
        // This CTA's 128 rows of A (of its problem) and half of the B rows, per slot.
        const int ma = r0.tm * BM + int(rank) * BMC, na = Ea.b_row0 + r0.tn * kTN + int(rank) * (kTN / 2);
        const int mb = r1.tm * BM + int(rank) * BMC, nb = Eb.b_row0 + r1.tn * kTN + int(rank) * (kTN / 2);
        // Main units, then the denoise units, in the issuer's order.  The two
        // loops are kept apart (and the tensor maps named, not selected), so
        // the per-stage code on the main path stays minimal.
        for (int u = 0; u < nmain && ok; ++u) {
          if (u == pf_unit && leader && t0 + stride < a.num_tiles) {
            // The next round's first K stages into L2, so its first units
            // do not wait a full HBM round trip right after the tile end
            // (where the ring has just held the denoise operands).
            const int t1 = t0 + stride;
            const bool two1 = a.tpr == 2 && t1 + 1 < a.num_tiles;
            for (int s = 0; s < (two1 ? 2 : 1); ++s) {
              const TileRef rn = item_of(a, x, t1 + s);
              const ExpertEntry& En = x.ex[rn.e];
              const int mn = rn.tm * BM + int(rank) * BMC;
              const int nn = En.b_row0 + rn.tn * kTN + int(rank) * (kTN / 2);
              for (int st = 0; st < pf_stages; ++st) {
                const int kx = rn.ks * nmain * unit_k + st * BK;
                tma_prefetch_l2_2d(&En.tmA, kx, mn);
                tma_prefetch_l2_2d(&a.tmB, kx, nn);
              }
            }
          }
          for (int s = 0; s < (two ? 2 : 1) && ok; ++s) {
            const int m0 = s ? mb : ma, n0 = s ? nb : na;
            const int kbase = (s ? r1.ks : r0.ks) * nmain;  // the item's K range (split-K), in units
            const CUtensorMap* tmA = s ? &Eb.tmA : &Ea.tmA;
            for (int st = 0; st < stages_per_unit; ++st, ++it) {
              const int j = it % kStages;
              if (!(ok = mbar_wait_warp(&S.empty[j], ((it / kStages) & 1) ^ 1, abort_flag, a.sync, a.wait_budget, a.wait_hint_ns))) break;
              uint8_t* sa = stage_mem + j * kStageBytes;
              const int kbyte = (kbase + u) * unit_k + st * BK;
              if (leader) {
                // The leader CTA's full barrier counts both CTAs' bytes.
                if (rank == 0) mbar_arrive_expect_tx(&S.full[j], 2 * kStageBytes);
                tma_load_2d_2sm(tmA, &S.full[j], sa, kbyte, m0);
                tma_load_2d_2sm(&a.tmB, &S.full[j], sa + kAStage, kbyte, n0);
              }
            }
          }
        }
        if (kDenoise) {
          for (int s = 0; s < (two ? 2 : 1) && ok; ++s) {
            for (int d = 0; d < nden && ok; ++d) {
              const int m0 = s ? mb : ma, n0 = s ? nb : na;
              const ExpertEntry& Es = s ? Eb : Ea;
              for (int st = 0; st < stages_per_unit; ++st, ++it) {
                const int j = it % kStages;
                if (!(ok = mbar_wait_warp(&S.empty[j], ((it / kStages) & 1) ^ 1, abort_flag, a.sync, a.wait_budget, a.wait_hint_ns))) break;
                uint8_t* sa = stage_mem + j * kStageBytes;
                const int ds = d * stages_per_unit + st;
                const int col = (ds % den_stages_per_product) * (BK / 2);
                if (leader) {
                  if (rank == 0) mbar_arrive_expect_tx(&S.full[j], 2 * kStageBytes);
                  if (ds < den_stages_per_product) {
                    tma_load_2d_2sm(&Es.tmDA0, &S.full[j], sa, col, m0);
                    tma_load_2d_2sm(&a.tmDB0, &S.full[j], sa + kAStage, col, n0);
                  } else {
                    tma_load_2d_2sm(&Es.tmDA1, &S.full[j], sa, col, m0);
                    tma_load_2d_2sm(&a.tmDB1, &S.full[j], sa + kAStage, col, n0);
                  }
                }
              }
            }
          }
        }
      }
      // Drain (bounded): every issued stage has been consumed by the MMAs,
      // hence has landed, before this CTA leaves.
      for (uint32_t j = (it > uint32_t(kStages) ? it - kStages : 0); j < it; ++j) {
        long long t0 = clock64();
        while (!mbar_test(&S.empty[j % kStages], (j / kStages) & 1) && clock64() - t0 < 100000000LL) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    // The whole warp runs the issue loop and one elected lane issues each
    // MMA and commit (the *_warp forms), so the loop state is warp-uniform.
    // The instruction stream is kept lean: the i8 and f16 MMAs sit in
    // separate loops and the accumulate flag is computed once per stage (a
    // runtime kind switch inside the unrolled MMA block measurably slows the
    // issue rate below the tensor pipe's).
    if (rank == 0) {
      uint32_t it = 0;
      uint32_t empar = 0;  // acc_empty parity per slot
      uint32_t pend = 0;   // bit s: slot s holds a unit the fold warps have not released yet
      bool ok = true;
      const uint32_t sbase = smem_u32(stage_mem);
      auto acquire = [&](int s) -> bool {
        if (!bit(pend, s)) return true;
        if (!mbar_wait_warp(&S.acc_empty[s], bit(empar, s), abort_flag, a.sync, a.wait_budget, a.wait_hint_ns)) return false;
        empar ^= 1u << s;
        pend &= ~(1u << s);
        tc_fence_after();
        return true;
      };
      auto main_unit = [&](int s, int u) {
        // Operands first (usually resident already), then the slot.
        if (!(ok = mbar_wait_warp(&S.full[it % kStages], (it / kStages) & 1, abort_flag, a.sync, a.wait_budget, a.wait_hint_ns))) return;
        if ((kReduce || u == 0) && !(ok = acquire(s))) return;
        const uint32_t dt = tmem + 256 * s;
        for (int st = 0; st < stages_per_unit; ++st, ++it) {
          const int j = it % kStages;
          if (st > 0 && !(ok = mbar_wait_warp(&S.full[j], (it / kStages) & 1, abort_flag, a.sync, a.wait_budget, a.wait_hint_ns))) return;
          tc_fence_after();
          const uint64_t ad = sdesc_kmajor<BK>(sbase + j * kStageBytes);
          const uint64_t bd = sdesc_kmajor<BK>(sbase + j * kStageBytes + kAStage);
          umma_8bit_2sm_stage_warp<BK / 32, (kKind != 0)>(dt, ad, bd, kIdescI8, uint32_t((u | st) != 0), &S.empty[j], kPairMask);
        }
        // With the transcript every unit is a fold event, and the stage's
        // commit above doubles as "accumulator ready" (one commit per unit
        // keeps the tensor pipe's queue full).  A tile's last unit gets its
        // own commit: its stage is refilled by the denoise units of the
        // other slot, which do not wait for this slot's event.
        if (u == nmain - 1) umma_commit_2sm_warp(&S.acc_full[s], kPairMask);
        if (kReduce || u == nmain - 1) pend |= 1u << s;
      };
      auto denoise_unit = [&](int s, int d) {
        if (d == 0 && !(ok = acquire(s))) return;  // S has been rewritten as f32
        const uint32_t dt = tmem + 256 * s;
        for (int st = 0; st < stages_per_unit; ++st, ++it) {
          const int j = it % kStages;
          if (!(ok = mbar_wait_warp(&S.full[j], (it / kStages) & 1, abort_flag, a.sync, a.wait_budget, a.wait_hint_ns))) return;
          tc_fence_after();
          const uint64_t ad = sdesc_kmajor<BK>(sbase + j * kStageBytes);
          const uint64_t bd = sdesc_kmajor<BK>(sbase + j * kStageBytes + kAStage);
#pragma unroll
          for (int ks = 0; ks < BK / 32; ++ks) umma_f16_2sm_warp(dt, ad + 2 * ks, bd + 2 * ks, kIdescF16, 1);
          umma_commit_2sm_warp(&S.empty[j], kPairMask);
        }
        if (d == nden - 1) {
          umma_commit_2sm_warp(&S.acc_full[s], kPairMask);
          pend |= 1u << s;
        }
      };
      for (int t0 = first; t0 < a.num_tiles && ok; t0 += stride) {
        const bool two = a.tpr == 2 && t0 + 1 < a.num_tiles;
        for (int u = 0; u < nmain && ok; ++u) {
          main_unit(0, u);
          if (two && ok) main_unit(1, u);
        }
        // Each slot's denoise units back to back: slot 0's run while the fold
        // warps still rewrite slot 1's accumulator as f32.
        if (kDenoise) {
          for (int d = 0; d < nden && ok; ++d) denoise_unit(0, d);
          if (two)
            for (int d = 0; d < nden && ok; ++d) denoise_unit(1, d);
        }
      }
      // Every MMA has retired before TMEM is released.
      umma_commit_2sm_warp(&S.drain, 0x1);
      long long t0 = clock64();
      while (!mbar_test(&S.drain, 0) && clock64() - t0 < 100000000LL) {
      }
    }
  } else if (warp < 2 + kFoldWarps) {
    // ------------------------------------------------------------ fold warps
    // Four warps per TMEM lane quadrant q = warp % 4 (the quadrant a warp may
    // access); warp index wi = 0..3 within the quadrant picks the 64-column
    // strip [64 wi, 64 wi + 64).  Loads use the 32x32b shape (thread = row),
    // which reads TMEM about twice as fast as the 16-lane shapes; both
    // 32-column loads of a strip are in flight before the wait.
    //
    // Fold of one R-chunk u: each thread XORs its row's strip values into the
    // four column classes (col / 2) % 4 of the hash tiles (rows r and r + 8
    // meet in the transcript word's atomics).  Word w = u % 16 of a transcript is rotated
    // by 13 at each later chunk with the same w, so the final transcript is
    // the XOR over chunks of rotl(fold_u, 13 * (later chunks on w)); the
    // rotation is linear, so every strip warp pre-rotates its partial fold
    // and XORs it into the tile's transcript word in shared memory with an
    // atomic -- no per-chunk combine or barrier.  Each slot has two
    // transcript buffers (alternating rounds); after a tile's last chunk the
    // hash warps take the buffer over while the slot's next tile fills the
    // other one.
    const int fw = warp - 2;
    const int q = warp & 3;
    const int wi = fw >> 2;
    const uint32_t strip_off = (uint32_t(32 * q) << 16) + 64 * wi;
    // Slot releases go to the leader's acc_empty (remotely from the peer).
    const uint32_t rel_base = mapa(&S.acc_empty[0], 0);
    // Transcript words this lane XORs into: row pair (lane % 8) + 8 (lane / 16)
    // of lane quadrant q, class c at + 16 c.
    const int lane_tile = q * 64 + (lane & 7) + 8 * (lane >> 4);
    uint32_t fpar = 0;  // acc_full parity per slot
    bool ok = true;

    // Transcript chunks (every main unit when kReduce) are final when the
    // commit that frees the unit's last operand stage fires: empty[] of that
    // stage, phase = stage count / kStages.  A parity wait is exact only if
    // the barrier has completed the phase before it -- true here, because
    // these warps waited for the slot's previous unit, which came later in
    // the issue order than the stage's previous use -- and if the phase
    // cannot be overtaken, which it cannot: the issuer reuses the slot, and
    // so comes within kStages units of refilling the stage, only after these
    // warps release it.  A tile's last chunk has no such guarantee (slot 0's
    // denoise units refill slot 1's last stage without waiting for slot 1's
    // event), so it and the final store wait on the slot's acc_full commit.
    auto fold_slot = [&](auto slot, int round, int u, const TileRef& tr, uint32_t last_stage) {
      const int tm = tr.tm, tn = tr.tn;
      const ExpertEntry& E = x.ex[tr.e];
      constexpr int s = decltype(slot)::value;
      const int b = 2 * s + (round & 1);  // transcript buffer
      const bool is_main = u < nmain;
      const bool last_main = u == nmain - 1;
      if (kReduce && is_main && !last_main) {
        if (!(ok = mbar_wait_warp(&S.empty[last_stage % kStages], (last_stage / kStages) & 1, abort_flag, a.sync,
                                  a.wait_budget, a.wait_hint_ns)))
          return;
      } else {
        if (!(ok = mbar_wait_warp(&S.acc_full[s], bit(fpar, s), abort_flag, a.sync, a.wait_budget, a.wait_hint_ns))) return;
        fpar ^= 1u << s;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + 256 * s + strip_off;
      const bool do_fold = kReduce && is_main;
      const bool do_convert = kDenoise && last_main;
      const bool do_store = (!kDenoise && last_main) || !is_main;
      // The strip is read as two 32-column halves (32 registers each): 64
      // live accumulators would not fit beside the rest of a fold warp's
      // state in the 96 registers 20 warps leave per thread, and spilled
      // registers go to a 29 KB L1 (the rest of the SM's SRAM is shared
      // memory).  The per-chunk fold and a tile's last events (f32 rewrite,
      // C) are separate code paths so the hot one stays small.
      auto release = [&](bool after_store) {
        // The slot's TMEM traffic is done.  After loads only (drained by
        // wait::ld) a relaxed arrive suffices, and it never waits for this
        // warp's C stores still in flight.  After the f32 rewrite the
        // tcgen05.st have completed (wait::st) and the tcgen05 fence orders
        // them before the arrive, which releases at CTA scope (the default
        // of a shared::cluster arrive).  A cluster-scope release here cost
        // ~2000 cycles per rewrite, measured, on the path the issuer waits on.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (after_store)
            mbar_arrive_cluster_addr(rel_base + 8 * s);
          else
            mbar_arrive_relaxed_cluster(rel_base + 8 * s);
        }
      };
      // XORs the pre-rotated class folds into the tile's four transcript
      // words (one per column class).  Rows r and r + 8 of a hash tile sit in
      // lanes l and l ^ 8, which XOR into the same words: the atomics pair
      // them, so no shuffle is needed (fewer instructions per event than a
      // shuffle-and-select pairing, on sub-partitions the issuer and the
      // producer share with these warps).
      auto commit_fold = [&](uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3) -> bool {
        const int w = u & 15;
        const int later = ((nmain - 1 - w) >> 4) - (u >> 4);  // chunks after u that hit word w
        const int rot = (13 * later) & 31;
        // A tile's first chunk reuses the buffer of two rounds ago: the hash
        // warps must have cleared it.
        if (u == 0 && round >= 2 &&
            !(ok = mbar_wait_idle_warp(&S.xfree[b], ((round >> 1) - 1) & 1, abort_flag, a.sync, a.wait_budget, a.wait_hint_ns)))
          return false;
        uint32_t* tw = xbuf + b * (16 * 256) + w * 256 + lane_tile;
        atomicXor(tw, __funnelshift_l(p0, p0, rot));
        atomicXor(tw + 16, __funnelshift_l(p1, p1, rot));
        atomicXor(tw + 32, __funnelshift_l(p2, p2, rot));
        atomicXor(tw + 48, __funnelshift_l(p3, p3, rot));
        // The reference counts one hash per 2 x 64 tile of each 128-row
        // tile that starts inside M.
        if (kDebug && lane == 0 && tm * BM + int(rank) * BMC < E.m) atomicAdd(a.counter, 16ull);
        if (last_main) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.xready[b]);  // this warp's contributions are in
        }
        return true;
      };
      auto fold32 = [](const uint32_t* v, uint32_t& p0, uint32_t& p1, uint32_t& p2, uint32_t& p3) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          p0 ^= v[i] ^ v[i + 1];
          p1 ^= v[i + 2] ^ v[i + 3];
          p2 ^= v[i + 4] ^ v[i + 5];
          p3 ^= v[i + 6] ^ v[i + 7];
        }
      };

      // The 16 words of class c in a 64-column strip (columns 8j + 2c and
      // 8j + 2c + 1 of both halves) as a depth-3 tree of 3-input XORs.
      auto class_fold = [](const uint32_t* a, const uint32_t* b, int c) -> uint32_t {
        const uint32_t t0 = a[2 * c] ^ a[2 * c + 1] ^ a[8 + 2 * c];
        const uint32_t t1 = a[9 + 2 * c] ^ a[16 + 2 * c] ^ a[17 + 2 * c];
        const uint32_t t2 = a[24 + 2 * c] ^ a[25 + 2 * c] ^ b[2 * c];
        const uint32_t t3 = b[2 * c + 1] ^ b[8 + 2 * c] ^ b[9 + 2 * c];
        const uint32_t t4 = b[16 + 2 * c] ^ b[17 + 2 * c] ^ b[24 + 2 * c];
        return (t0 ^ t1 ^ t2) ^ (t3 ^ t4 ^ b[25 + 2 * c]);
      };

      if (!do_convert && !do_store) {
        // ---- every chunk but a tile's last: fold only
        uint32_t v0[32], v1[32];
        __syncwarp();
        tmem_ld32(taddr, v0);  // both halves in flight, one wait
        tmem_ld32(taddr + 32, v1);
        tmem_wait_ld_into2(v0, v1);
        release(false);
        commit_fold(class_fold(v0, v1, 0), class_fold(v0, v1, 1), class_fold(v0, v1, 2), class_fold(v0, v1, 3));
        return;
      }
      // ---- a tile's last chunk (fold + f32 rewrite, or fold + C) or its final C.
      // Both paths give the slot back as soon as its TMEM has been read (or
      // rewritten): the issuer waits for that release before the denoise
      // MMAs or the slot's next tile, and both slots reach their tile ends
      // together, so the tensor pipe idles for as long as this takes.
      uint32_t p0 = 0, p1 = 0, p2 = 0, p3 = 0;
      // With 128-wide tiles the strips beyond the tile hold nothing to store.
      const bool strip_live = 64 * wi < kTN;
      if (do_convert) {
        // Both halves in flight (as in the fold-only path), one load wait,
        // one store wait: S as f32 * 2^-12 for the f16 denoise MMAs (folded
        // first).
        if (strip_live) {
          uint32_t v0[32], v1[32];
          __syncwarp();
          tmem_ld32(taddr, v0);
          tmem_ld32(taddr + 32, v1);
          tmem_wait_ld_into(v0);
          tmem_wait_ld_into(v1);
          if (do_fold) {
            fold32(v0, p0, p1, p2, p3);
            fold32(v1, p0, p1, p2, p3);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) v0[i] = __float_as_uint(float(int(v0[i])) * (1.0f / 4096.0f));
          tmem_st32(taddr, v0);
#pragma unroll
          for (int i = 0; i < 32; ++i) v1[i] = __float_as_uint(float(int(v1[i])) * (1.0f / 4096.0f));
          tmem_st32(taddr + 32, v1);
          tmem_wait_st();
        }
        release(true);
        if (do_fold) commit_fold(p0, p1, p2, p3);
        return;
      }
      // C: the halves are read one at a time (one 32-column half live: a
      // spill-free kernel at 96 registers).  The first half goes into the
      // warp's shared-memory box and out by TMA before the second is read;
      // the slot is released right after the second read, so the second
      // box write -- which waits for the first TMA store to have read the
      // box -- is off the release path.
      float rs = 0.f;
      float2 sbv = make_float2(0.f, 0.f);
      {  // scales first: their latency overlaps the loads
        const int row = tm * BM + int(rank) * BMC + 32 * q + lane;
        rs = (row < E.m ? E.sA[a.scale_per_tensor ? 0 : row] : 0.0f) * (is_main ? 1.0f : 4096.0f);
        const int c = tn * kTN + 64 * wi + 2 * lane;  // this lane's two column scales
        if (c < a.N)
          sbv = a.scale_per_tensor ? make_float2(E.sB[0], E.sB[0]) : *reinterpret_cast<const float2*>(E.sB + c);
      }
      auto pack_half = [&](const uint32_t* v, int h, uint32_t* packed) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int src = 16 * h + i / 2;  // lane holding columns 32h + i, +1
          const float bx = __shfl_sync(0xffffffffu, sbv.x, src);
          const float by = __shfl_sync(0xffffffffu, sbv.y, src);
          const float f0 = (is_main && kKind == 0) ? float(int(v[i])) : __uint_as_float(v[i]);
          const float f1 = (is_main && kKind == 0) ? float(int(v[i + 1])) : __uint_as_float(v[i + 1]);
          packed[i / 2] = pack_bf16(f0 * rs * bx, f1 * rs * by);
        }
      };
      if (strip_live && !kReduce && !kDenoise && a.ksplit > 1) {
        // A split-K item: this warp's 32 x 64 block of the exact int32
        // partial goes to ws[ks] as it is; the reduction kernel sums the
        // ranges and scales.  After the CTA's last item the operand ring is
        // idle (every stage has been consumed by the MMAs this event waited
        // for), so the block is staged there as four 16-column boxes and
        // leaves by TMA stores (whole lines, rows >= m clipped within the
        // slab); otherwise it is stored from registers, 16 bytes per lane.
        const int row0 = tm * BM + int(rank) * BMC + 32 * q;
        const int row = row0 + lane;
        const bool staged = kRingStagesPartials && first + (round + 1) * stride >= a.num_tiles;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(taddr + 32 * h, v);
          tmem_wait_ld_into(v);
          if (h == 1) release(false);
          const int col = tn * kTN + 64 * wi + 32 * h;
          if (staged) {
#pragma unroll
            for (int p = 0; p < 2; ++p) {
              uint8_t* box = stage_mem + fw * 8192 + (2 * h + p) * 2048;
              uint8_t* rowp = box + lane * 64;
#pragma unroll
              for (int k = 0; k < 4; ++k)
                *reinterpret_cast<uint4*>(rowp + ((k ^ ((lane >> 1) & 3)) << 4)) =
                    make_uint4(v[16 * p + 4 * k], v[16 * p + 4 * k + 1], v[16 * p + 4 * k + 2], v[16 * p + 4 * k + 3]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_3d(&a.tmW, box, col + 16 * p, row0, tr.ks);
                bulk_commit_group();
              }
            }
          } else if (row < E.m) {
            int32_t* dst = a.ws + (int64_t(tr.ks) * E.m + row) * int64_t(a.N) + col;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (col + 4 * j < a.N)
                *reinterpret_cast<uint4*>(dst + 4 * j) = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
        }
      } else if (strip_live) {
        const int row0 = tm * BM + int(rank) * BMC + 32 * q;
        uint8_t* box = cstage + fw * kCBoxBytes;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v[32], pk[16];
          __syncwarp();
          tmem_ld32(taddr + 32 * h, v);
          tmem_wait_ld_into(v);
          if (do_fold) fold32(v, p0, p1, p2, p3);
          if (h == 1) release(false);
          pack_half(v, h, pk);
          if (kE > 1 && E.c_rows) {
            // Row map: the block goes through the warp's shared-memory box
            // (as for the TMA store) and out in whole 64-byte rows, eight
            // rows per store instruction (four lanes a row), each to the row
            // the map names; rows outside the destination are skipped.
            const int row = row0 + lane;
            const long long my_dr = row < E.m ? (long long)E.c_rows[row] : -1;
            const int col = tn * kTN + 64 * wi + 32 * h;
            uint8_t* rowp = box + lane * 64;
            __syncwarp();  // the box's previous rows have been read
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              *reinterpret_cast<uint4*>(rowp + ((kk ^ ((lane >> 1) & 3)) << 4)) =
                  make_uint4(pk[4 * kk], pk[4 * kk + 1], pk[4 * kk + 2], pk[4 * kk + 3]);
            __syncwarp();
            const int piece = lane & 3;
#pragma unroll
            for (int it = 0; it < 4; ++it) {
              const int br = 8 * it + (lane >> 2);  // box row this lane moves
              const long long dr = __shfl_sync(0xffffffffu, my_dr, br);
              const uint4 val = *reinterpret_cast<const uint4*>(box + br * 64 + ((piece ^ ((br >> 1) & 3)) << 4));
              if (dr >= 0 && dr < a.c_dst_rows && col + 8 * piece < a.N)
                *reinterpret_cast<uint4*>(a.c_dst + dr * a.N + col + 8 * piece) = val;
            }
          } else {
            store_c_packed(&E.tmC, box, pk, row0, tn * kTN + 64 * wi + 32 * h, lane);
          }
        }
      } else {
        release(false);
      }
      if (do_fold) commit_fold(p0, p1, p2, p3);
    };

    uint32_t it = 0;  // operand stages issued so far, in the issuer's order
    for (int t0 = first; t0 < a.num_tiles && ok; t0 += stride) {
      const bool two = a.tpr == 2 && t0 + 1 < a.num_tiles;
      const TileRef r0 = item_of(a, x, t0);
      const TileRef r1 = two ? item_of(a, x, t0 + 1) : r0;
      const int round = (t0 - first) / stride;
      for (int u = 0; u < units && ok; ++u) {
        const bool is_main = u < nmain;
        const bool event = (is_main && (kReduce || u == nmain - 1)) || (!is_main && u == units - 1);
        const uint32_t it0 = it;
        it += uint32_t((two ? 2 : 1) * stages_per_unit);
        if (!event) continue;
        fold_slot(I0{}, round, u, r0, it0 + stages_per_unit - 1);
        if (two && ok) fold_slot(I1{}, round, u, r1, it0 + 2 * stages_per_unit - 1);
      }
    }
    if (lane == 0) bulk_wait_all();  // C is written before the kernel ends
  } else if (kReduce) {
    // ------------------------------------------------------------ hash warps
    // Thread j hashes tiles j + 64 i (i < 4) of a finished transcript buffer;
    // tile q * 64 + c * 16 + p is row pair p (rows 32 q + (p % 8) + 16 (p / 8)
    // and +8) of lane quadrant q, column class c.  Each word is cleared after
    // it is read, for the slot's tile two rounds later.
    const int j = (warp - 2 - kFoldWarps) * 32 + lane;
    bool ok = true;
    auto hash_buffer = [&](auto slot, int round, const TileRef& tr) {
      const int tm = tr.tm, tn = tr.tn;
      const ExpertEntry& E = x.ex[tr.e];
      const int b = 2 * decltype(slot)::value + (round & 1);
      if (!(ok = mbar_wait_idle_warp(&S.xready[b], (round >> 1) & 1, abort_flag, a.sync, a.wait_budget, a.wait_hint_ns))) return;
      const int tm128 = 2 * tm + int(rank);
#pragma unroll 1
      for (int i = 0; i < 4; ++i) {
        const int ht = j + 64 * i;
        uint32_t* tr = xbuf + b * (16 * 256) + ht;
        uint32_t T[16], key[8], dg[8];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          T[k] = tr[k * 256];
          tr[k * 256] = 0u;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) key[k] = a.key[k];
        b3_compress8(key, T, kB3SingleBlockKeyed, dg);
        const int hq = ht >> 6, cls = (ht >> 4) & 3, p = ht & 15;
        const int row_in_tile = 32 * hq + (p & 7) + 16 * (p >> 3);
        const int64_t grow = int64_t(tm128) * BMC + row_in_tile;
        const int64_t gcol = int64_t(tn) * BN + 2 * cls;
        const bool in_bounds = (grow + 8 < E.m) && (gcol + 249 < a.N);
        if (in_bounds && (E.transcripts || E.digests)) {
          const int64_t idx = (grow / 16 * 8 + grow % 16) * (a.N / 64) + gcol / 256 * 4 + (gcol % 256) / 2;
          if (E.transcripts)
            for (int k = 0; k < 16; ++k) E.transcripts[idx * 16 + k] = T[k];
          if (E.digests)
            for (int k = 0; k < 8; ++k) E.digests[idx * 8 + k] = dg[k];
        }
        if (in_bounds && u256_le(dg, a.target)) publish_hit(a, E, tm128, tn, row_in_tile, cls, dg);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.xfree[b]);
    };
    for (int t0 = first; t0 < a.num_tiles && ok; t0 += stride) {
      const bool two = a.tpr == 2 && t0 + 1 < a.num_tiles;
      const int round = (t0 - first) / stride;
      const TileRef r0 = item_of(a, x, t0);
      const TileRef r1 = two ? item_of(a, x, t0 + 1) : r0;
      hash_buffer(I0{}, round, r0);
      if (two && ok) hash_buffer(I1{}, round, r1);
    }
  }

  // Neither CTA leaves while its peer can still address its barriers or TMEM.
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_2sm(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host
// CTA pairs of the mined-GEMM kernels resident at once on `device` (SM pairs
// in one GPC; 0 until the first launch there has asked the occupancy API).
int& resident_pairs(int device) {
  static int cached[64] = {0};
  return cached[device & 63];
}

template <int BK, int SPU, bool R_, bool D_, bool G_, int TN, int kE, int kKind = 0>
int launch_variant(const MainArgs& a, const ExpertTable<kE>& x, int device, cudaStream_t s) {
  auto kern = noisy_gemm_kernel<BK, SPU, R_, D_, G_, TN, kE, kKind>;
  const int smem = stage_budget(R_) + (R_ ? kXbufBytes : 0) + kCStageBytes + int(sizeof(Smem)) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status();
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // A persistent grid: as many CTA pairs as can be co-resident (SM pairs in
  // one GPC), never more than the tiles need (a pair runs tpr per round).
  int resident = resident_pairs(device);
  if (resident == 0) {
    cfg.gridDim = dim3(2, 1, 1);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      const int sms = sm_count(device);
      clusters = (sms > 0 ? sms : 148) / 2;
    }
    resident = clusters;
    resident_pairs(device) = clusters;
  }
  const int pairs = std::max(1, std::min((a.num_tiles + a.tpr - 1) / a.tpr, resident));
  cfg.gridDim = dim3(unsigned(2 * pairs), 1, 1);
  cudaLaunchAttribute attrs[2] = {attr[0], {}};
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddep_wait
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, kern, a, x);
  return launch_status();
}

template <int BK, int SPU>
int launch_spu(const MainArgs& a, const ExpertTable<1>& x, int device, bool reduce, bool denoise, bool debug,
               bool narrow, cudaStream_t s) {
  if (narrow) return launch_variant<BK, SPU, false, false, false, BN / 2, 1>(a, x, device, s);
  if (reduce && denoise) return debug ? launch_variant<BK, SPU, true, true, true, BN, 1>(a, x, device, s)
                                      : launch_variant<BK, SPU, true, true, false, BN, 1>(a, x, device, s);
  if (reduce) return debug ? launch_variant<BK, SPU, true, false, true, BN, 1>(a, x, device, s)
                           : launch_variant<BK, SPU, true, false, false, BN, 1>(a, x, device, s);
  if (denoise) return launch_variant<BK, SPU, false, true, false, BN, 1>(a, x, device, s);
  return launch_variant<BK, SPU, false, false, false, BN, 1>(a, x, device, s);
}

// The A-side tensor maps and scalars of one problem: rows [0, m) of the
// A-side arrays starting at the given pointers.
int make_entry(ExpertEntry& e, const void* ApEA, const void* EAL_fp16, const void* AxEBL_fp16, const float* sA,
               void* C, int64_t m, int64_t n, int64_t k, int64_t r, int bk, bool denoise) {
  const CUtensorMapSwizzle swz = bk == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  int st;
  if ((st = make_tmap_2d(&e.tmA, ApEA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, m, bk, BMC, swz))) return st;
  if ((st = make_tmap_2d(&e.tmC, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, m, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  if (denoise) {
    const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int dc = bk / 2;  // fp16 elements per stage row
    if ((st = make_tmap_2d(&e.tmDA0, EAL_fp16, F16, 2, r, m, dc, BMC, swz)) ||
        (st = make_tmap_2d(&e.tmDA1, AxEBL_fp16, F16, 2, r, m, dc, BMC, swz)))
      return st;
  }
  e.m = int(m);
  e.tiles_m = int((m + BM - 1) / BM);
  e.sA = sA;
  return PB2_OK;
}

bool al16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// The launch-wide arguments: B-side tensor maps (n rows per problem; the
// grouped launch passes all problems' rows in one array), shapes and the
// hash inputs.
int make_shared_args(MainArgs& a, const pb2_gemm_params& p, int bk, int tn_width, bool denoise,
                     int64_t b_rows = -1) {
  if (b_rows < 0) b_rows = p.n;
  const CUtensorMapSwizzle swz = bk == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  int st;
  if ((st = make_tmap_2d(&a.tmB, p.BpEB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.k, b_rows, bk, tn_width / 2, swz)))
    return st;
  if (denoise) {
    const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int dc = bk / 2;
    if ((st = make_tmap_2d(&a.tmDB0, p.EARxBpEB_fp16, F16, 2, p.r, b_rows, dc, BN / 2, swz)) ||
        (st = make_tmap_2d(&a.tmDB1, p.EBR_fp16, F16, 2, p.r, b_rows, dc, BN / 2, swz)))
      return st;
  }
  a.N = int(p.n);
  a.K = int(p.k);
  a.R = int(p.r);
  a.tiles_n = int((p.n + tn_width - 1) / tn_width);
  a.group = p.swizzle > 0 ? p.swizzle : 8;
  a.target = p.pow_target;
  a.key = p.pow_key;
  a.counter = reinterpret_cast<unsigned long long*>(p.inner_hash_counter);
  a.wait_budget = wait_budget_cycles();
  a.wait_hint_ns = suspend_hint_ns(a.wait_budget);
  return PB2_OK;
}

// The K split of a plain GEMM whose 256 x 256 tiles are too few to fill the
// SM pairs (a decode batch): the largest d <= 4 that divides K's 128-byte
// units into ranges of at least kMinSplitUnits units and keeps tiles x d work
// items within one round of pairs.  1: no split.  A split costs a write and
// a read of d int32 partials of C and a second launch (measured ~8 us at
// m = 256, n = 4096), so only long K ranges (the down projection's 14336)
// gain from it.
constexpr int64_t kMinSplitUnits = 24;
int splitk_plan(int device, int64_t m, int64_t n, int64_t k) {
  const int64_t tiles = ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
  const int pairs = resident_pairs(device) ? resident_pairs(device) : std::max(1, sm_count(device) / 2);
  const int64_t units = k / kTileK;
  if (tiles >= pairs || k % kTileK != 0) return 1;
  int best = 1;
  for (int d = 2; d <= 4; ++d)
    if (units % d == 0 && units / d >= kMinSplitUnits && tiles * d <= pairs) best = d;
  return best;
}

// C = bf16(float(sum over the K ranges of the int32 partials) * sA * sB), the
// epilogue's arithmetic in its order; one thread per 8 columns.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const int32_t* ws, int ksplit, int64_t m, int64_t n,
                                                            const float* sA, const float* sB, int per_tensor,
                                                            __nv_bfloat16* C) {
  griddep_wait();  // launched behind the GEMM (programmatic dependent launch)
  griddep_launch_dependents();
  const int64_t vecs = n / 8;
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= m * vecs) return;
  const int64_t row = i / vecs, col = (i - row * vecs) * 8;
  int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int s = 0; s < ksplit; ++s) {
    const int4* p = reinterpret_cast<const int4*>(ws + (int64_t(s) * m + row) * n + col);
    const int4 x = p[0], y = p[1];
    acc[0] += x.x; acc[1] += x.y; acc[2] += x.z; acc[3] += x.w;
    acc[4] += y.x; acc[5] += y.y; acc[6] += y.z; acc[7] += y.w;
  }
  const float ra = sA[per_tensor ? 0 : row];
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    const float b0 = sB[per_tensor ? 0 : col + j], b1 = sB[per_tensor ? 0 : col + j + 1];
    out[j / 2] = pack_bf16(float(acc[j]) * ra * b0, float(acc[j + 1]) * ra * b1);
  }
  *reinterpret_cast<uint4*>(C + row * n + col) = make_uint4(out[0], out[1], out[2], out[3]);
}

int launch_splitk_reduce(const int32_t* ws, int ksplit, int64_t m, int64_t n, const float* sA, const float* sB,
                         void* C, cudaStream_t s) {
  const int64_t threads = m * (n / 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((threads + 255) / 256), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, ws, ksplit, m, n, sA, sB, 0, static_cast<__nv_bfloat16*>(C));
  return launch_status();
}

}  // namespace

// Every check of the main kernel's arguments that needs no CUDA call.
int check_main_args(const pb2_gemm_params& p, bool reduce, bool denoise) {
  if (p.m <= 0 || p.n <= 0 || p.k <= 0) return PB2_ERR_INVALID_ARGUMENT;
  if (p.tile_size_m != BMC || p.tile_size_n != BN || p.tile_size_k != kTileK) return PB2_ERR_UNSUPPORTED_CONFIG;
  if (p.cluster_size_m != 1 || p.cluster_size_n != 1) return PB2_ERR_UNSUPPORTED_CONFIG;
  // pipeline_stages is a hint: the ring depth is fixed by the shared-memory plan.
  if (p.k % kTileK != 0 || p.n % 8 != 0) return PB2_ERR_INVALID_ARGUMENT;
  if (p.m > INT32_MAX || p.n > INT32_MAX || p.k > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  if ((reduce || denoise) && !(p.r == 64 || p.r == 128 || p.r == 256)) return PB2_ERR_UNSUPPORTED_CONFIG;
  if ((reduce || denoise) && (p.k % p.r != 0)) return PB2_ERR_INVALID_ARGUMENT;
  if (!p.ApEA || !p.BpEB || !p.A_scales || !p.B_scales || !p.C) return PB2_ERR_INVALID_ARGUMENT;
  if (!al16(p.ApEA) || !al16(p.BpEB) || !al16(p.C) || !al16(p.B_scales)) return PB2_ERR_INVALID_ARGUMENT;
  if (reduce && (!p.host_signal_sync || !p.pow_target || !p.pow_key)) return PB2_ERR_INVALID_ARGUMENT;
  if (denoise && (!p.EAL_fp16 || !p.EBR_fp16 || !p.AxEBL_fp16 || !p.EARxBpEB_fp16))
    return PB2_ERR_INVALID_ARGUMENT;
  if (reduce && p.enable_debug && !p.inner_hash_counter) return PB2_ERR_INVALID_ARGUMENT;
  if ((p.transcripts || p.digests) && (p.m % 16 != 0 || p.n % 256 != 0)) return PB2_ERR_INVALID_ARGUMENT;
  return PB2_OK;
}

// Every argument check of pb2_noisy_gemm that needs no CUDA call: a call
// these reject has queued no work.
int check_noisy_gemm_args(const pb2_gemm_params& p) {
  if (p.run_noising_a && (!p.A || !p.EAL || !p.EAR_R_major || !p.EBL_K_major)) return PB2_ERR_INVALID_ARGUMENT;
  if (p.run_noising_b && (!p.B || !p.EBR || !p.EAR_K_major || !p.EBL_R_major)) return PB2_ERR_INVALID_ARGUMENT;
  return check_main_args(p, !p.skip_reduction, !p.skip_denoising);
}

int run_main_kernel(const pb2_gemm_params& p, bool reduce, bool denoise, cudaStream_t s) {
  int cst = check_main_args(p, reduce, denoise);
  if (cst) return cst;
  const bool debug = reduce && p.enable_debug;

  // 128-byte stages (128-byte swizzle) unless R = 64, where 64-byte stages
  // (64-byte swizzle) keep a transcript chunk a whole number of stages.
  const int bk = ((reduce || denoise) && p.r == 64) ? 64 : 128;
  // The plain GEMM of a small problem (fewer 256-wide tiles than SM pairs,
  // e.g. a decode batch) runs 128-wide tiles: more SMs streaming the weights
  // (a 128-wide tile issues half the MMA work per instruction, so wider
  // problems keep 256-wide tiles).  A plain GEMM whose tiles fit one round
  // of pairs runs one tile per pair.
  const int64_t tiles_m = (p.m + BM - 1) / BM;
  const int pairs_est = resident_pairs(p.device) ? resident_pairs(p.device) : std::max(1, sm_count(p.device) / 2);
  // A plain GEMM with too few 256 x 256 tiles splits K when the caller gave
  // the workspace; otherwise small problems take 128-wide tiles.
  int ksplit = 1;
  if (!reduce && !denoise && p.workspace) {
    ksplit = splitk_plan(p.device, p.m, p.n, p.k);
    if (ksplit > 1 && (p.workspace_bytes < int64_t(ksplit) * p.m * p.n * 4 || !al16(p.workspace))) ksplit = 1;
  }
  const bool narrow = ksplit == 1 && !reduce && !denoise && tiles_m * ((p.n + BN - 1) / BN) < int64_t(pairs_est);
  const int tn_width = narrow ? BN / 2 : BN;
  MainArgs a;
  std::memset(&a, 0, sizeof(a));
  ExpertTable<1> x;
  std::memset(&x, 0, sizeof(x));
  int st;
  if ((st = make_shared_args(a, p, bk, tn_width, denoise))) return st;
  if ((st = make_entry(x.ex[0], p.ApEA, p.EAL_fp16, p.AxEBL_fp16, p.A_scales, p.C, p.m, p.n, p.k, p.r, bk,
                       denoise)))
    return st;
  x.count = 1;
  ExpertEntry& e = x.ex[0];
  e.tile_begin = 0;
  e.b_row0 = 0;
  e.sB = p.B_scales;
  e.sync = static_cast<SignalSync*>(p.host_signal_sync);
  e.header = static_cast<SignalHeader*>(p.host_signal_header_pinned);
  e.hits = p.hits;
  e.hit_cap = p.hits ? p.hit_capacity : 0;
  e.transcripts = p.transcripts;
  e.digests = p.digests;
  a.num_tiles = e.tiles_m * a.tiles_n * ksplit;  // work items
  a.tpr = (!reduce && !denoise && a.num_tiles <= pairs_est) ? 1 : 2;
  a.ksplit = ksplit;
  a.ws = ksplit > 1 ? p.workspace : nullptr;
  if (ksplit > 1 && (st = make_tmap_3d(&a.tmW, p.workspace, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, p.n, p.m, ksplit, 16, 32,
                                       CU_TENSOR_MAP_SWIZZLE_64B)))
    return st;
  a.sync = e.sync;

  // Operand stages per unit: a unit is R bytes of K with transcript or
  // denoise (R = 64: one 64-byte stage; R = 128: one; R = 256: two), else
  // one 128-byte tile_size_k.
  const int spu = (reduce || denoise) ? int(p.r) / bk : kTileK / bk;
  if (bk == 64) return launch_spu<64, 1>(a, x, p.device, reduce, denoise, debug, false, s);
  st = spu == 2 ? launch_spu<128, 2>(a, x, p.device, reduce, denoise, debug, false, s)
                : launch_spu<128, 1>(a, x, p.device, reduce, denoise, debug, narrow, s);
  if (st || ksplit == 1) return st;
  return launch_splitk_reduce(p.workspace, ksplit, p.m, p.n, p.A_scales, p.B_scales, p.C, s);
}

// The mined GEMMs of several problems that share B's K-side noise and the
// hash inputs -- the experts of a MoE layer -- in persistent launches of up
// to kMaxExperts problems each.  Problem e reads rows [a_row0_e, a_row0_e +
// m_e) of the A-side arrays (ApEA, EAL_fp16, AxEBL_fp16, A_scales, C) and rows
// [e n, e n + n) of the B-side ones (BpEB, EARxBpEB_fp16, EBR_fp16,
// B_scales), and signals its hits through its own buffers.
int run_grouped_kernel(const pb2_gemm_params& p, const pb2_expert_gemm* experts, int64_t num_experts,
                       const int32_t* c_row_index, int64_t c_rows, cudaStream_t s) {
  const int bk = p.r == 64 ? 64 : 128;
  const int spu = int(p.r) / bk;
  for (int64_t e0 = 0; e0 < num_experts; e0 += kMaxExperts) {
    const int cnt = int(std::min<int64_t>(kMaxExperts, num_experts - e0));
    MainArgs a;
    std::memset(&a, 0, sizeof(a));
    ExpertTable<kMaxExperts> x;
    std::memset(&x, 0, sizeof(x));
    int st;
    if ((st = make_shared_args(a, p, bk, BN, true, num_experts * p.n))) return st;
    int tiles = 0;
    SignalSync* first_sync = nullptr;
    for (int i = 0; i < cnt; ++i) {
      const pb2_expert_gemm& q = experts[e0 + i];
      ExpertEntry& e = x.ex[i];
      e.tile_begin = tiles;
      e.b_row0 = int((e0 + i) * p.n);
      e.sB = p.B_scales + (e0 + i) * p.n;
      if (q.m > 0) {
        const int64_t r0 = q.a_row0;
        if ((st = make_entry(e, p.ApEA + r0 * p.k, static_cast<const uint16_t*>(p.EAL_fp16) + r0 * p.r,
                             static_cast<uint16_t*>(p.AxEBL_fp16) + r0 * p.r, p.A_scales + r0,
                             static_cast<uint16_t*>(p.C) + r0 * p.n, q.m, p.n, p.k, p.r, bk, true)))
          return st;
      }
      e.sync = static_cast<SignalSync*>(q.host_signal_sync);
      e.header = static_cast<SignalHeader*>(q.host_signal_header_pinned);
      e.hits = q.hits;
      e.hit_cap = q.hits ? q.hit_capacity : 0;
      e.transcripts = q.transcripts;
      e.digests = q.digests;
      e.c_rows = c_row_index && q.m > 0 ? c_row_index + q.a_row0 : nullptr;
      if (!first_sync && q.m > 0) first_sync = e.sync;
      tiles += e.tiles_m * a.tiles_n;
    }
    if (tiles == 0) continue;
    x.count = cnt;
    a.num_tiles = tiles;
    a.tpr = 2;
    a.sync = first_sync;
    a.c_dst = static_cast<uint16_t*>(p.C);
    a.c_dst_rows = c_row_index ? c_rows : 0;
    int dev = p.device;
    if (bk == 64) st = launch_variant<64, 1, true, true, false, BN, kMaxExperts>(a, x, dev, s);
    else if (spu == 2) st = launch_variant<128, 2, true, true, false, BN, kMaxExperts>(a, x, dev, s);
    else st = launch_variant<128, 1, true, true, false, BN, kMaxExperts>(a, x, dev, s);
    if (st) return st;
  }
  return PB2_OK;
}

int denoise_convert(const int32_t* in, void* out, int64_t count, float scale, cudaStream_t s);
int run_grouped_kernel(const pb2_gemm_params& p, const pb2_expert_gemm* experts, int64_t num_experts,
                       const int32_t* c_row_index, int64_t c_rows, cudaStream_t s);
int run_noising_both(const pb2_noising_params& pa, const pb2_noising_params& pb, cudaStream_t stream);

}  // namespace pb2

extern "C" int pb2_noisy_gemm(const pb2_gemm_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_noisy_gemm");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_gemm_params& p = *pp;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = check_noisy_gemm_args(p);
  if (st) return st;
  if ((st = set_device(p.device))) return st;
  pb2_noising_params qa{}, qb{};
  if (p.run_noising_a) {
    if (!p.A || !p.EAL || !p.EAR_R_major || !p.EBL_K_major) return PB2_ERR_INVALID_ARGUMENT;
    qa.device = p.device; qa.rows = p.m; qa.k = p.k; qa.r = p.r;
    qa.X = p.A; qa.EL = p.EAL; qa.E_rmajor = p.EAR_R_major; qa.E_kmajor = p.EBL_K_major;
    qa.XpE = p.ApEA;
    qa.proj = p.AxEBL_int32 ? static_cast<void*>(p.AxEBL_int32) : p.AxEBL_fp16;
    qa.proj_is_fp16 = p.AxEBL_int32 ? 0 : 1;
    qa.k_blocks_per_split = p.AxEBL_int32 ? p.k_blocks_per_split_noising_a : 0;
    qa.host_signal_sync = p.host_signal_sync;
  }
  if (p.run_noising_b) {
    if (!p.B || !p.EBR || !p.EAR_K_major || !p.EBL_R_major) return PB2_ERR_INVALID_ARGUMENT;
    qb.device = p.device; qb.rows = p.n; qb.k = p.k; qb.r = p.r;
    qb.X = p.B; qb.EL = p.EBR; qb.E_rmajor = p.EBL_R_major; qb.E_kmajor = p.EAR_K_major;
    qb.XpE = p.BpEB;
    qb.proj = p.EARxBpEB_int32 ? static_cast<void*>(p.EARxBpEB_int32) : p.EARxBpEB_fp16;
    qb.proj_is_fp16 = p.EARxBpEB_int32 ? 0 : 1;
    qb.k_blocks_per_split = p.EARxBpEB_int32 ? p.k_blocks_per_split_noising_b : 0;
    qb.host_signal_sync = p.host_signal_sync;
  }
  if (p.run_noising_a && p.run_noising_b) {
    if ((st = run_noising_both(qa, qb, s))) return st;
  } else if (p.run_noising_a) {
    if ((st = pb2_noise_A(&qa, stream))) return st;
  } else if (p.run_noising_b) {
    if ((st = pb2_noise_B(&qb, stream))) return st;
  }
  if (!p.skip_denoising) {
    if (p.AxEBL_int32 && (st = denoise_convert(p.AxEBL_int32, p.AxEBL_fp16, p.m * p.r, 1.0f / 16384.0f, s)))
      return st;
    if (p.EARxBpEB_int32 &&
        (st = denoise_convert(p.EARxBpEB_int32, p.EARxBpEB_fp16, p.n * p.r, 1.0f / 4096.0f, s)))
      return st;
  }
  return run_main_kernel(p, !p.skip_reduction, !p.skip_denoising, s);
}

extern "C" int pb2_gemm(const pb2_gemm_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_gemm");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(pp->device);
  if (st) return st;
  return run_main_kernel(*pp, false, false, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t pb2_gemm_workspace_bytes(int device, int64_t m, int64_t n, int64_t k) {
  using namespace pb2;
  if (m <= 0 || n <= 0 || k <= 0 || device < 0) return 0;
  const int d = splitk_plan(device, m, n, k);
  return d > 1 ? int64_t(d) * m * n * 4 : 0;
}

extern "C" int pb2_noisy_gemm_grouped(const pb2_grouped_gemm_params* gp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_noisy_gemm_grouped");
  using namespace pb2;
  if (!gp || !gp->experts || gp->num_experts <= 0) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_gemm_params& p = gp->shared;
  const int64_t E = gp->num_experts;
  if (p.skip_reduction || p.skip_denoising || p.enable_debug) return PB2_ERR_UNSUPPORTED_CONFIG;
  if (p.AxEBL_int32 || p.EARxBpEB_int32) return PB2_ERR_UNSUPPORTED_CONFIG;  // half projections only
  // The expert row ranges tile [0, p.m) in order, without gaps or overlap.
  int64_t next = 0;
  for (int64_t i = 0; i < E; ++i) {
    const pb2_expert_gemm& q = gp->experts[i];
    if (q.m < 0 || q.a_row0 != next) return PB2_ERR_INVALID_ARGUMENT;
    if (q.m > 0 && (!q.host_signal_sync || (q.a_row0 * p.k) % 16 || (q.a_row0 * p.n * 2) % 16 ||
                    (q.a_row0 * p.r * 2) % 16))
      return PB2_ERR_INVALID_ARGUMENT;
    if ((q.transcripts || q.digests) && (q.m % 16 != 0 || p.n % 256 != 0)) return PB2_ERR_INVALID_ARGUMENT;
    next += q.m;
  }
  if (next != p.m) return PB2_ERR_INVALID_ARGUMENT;
  // A row map sends C's rows into a destination of c_rows >= m rows (the
  // per-expert tensor maps, unused then, still cover rows [0, m) of it).
  if (gp->c_row_index && (gp->c_rows < p.m || reinterpret_cast<uintptr_t>(gp->c_row_index) % 4))
    return PB2_ERR_INVALID_ARGUMENT;
  // The shared checks on the stacked problem (all rows of A, n rows of B
  // per expert): a rejected call queues no work.
  pb2_gemm_params all = p;
  all.host_signal_sync = gp->experts[0].host_signal_sync ? gp->experts[0].host_signal_sync : &all;
  all.hits = nullptr;
  all.transcripts = nullptr;
  all.digests = nullptr;
  int st = check_noisy_gemm_args(all);
  if (st) return st;
  if (E * p.n > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  if ((st = set_device(p.device))) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Noising: row-independent, so one noise_A over every expert's rows and
  // one noise_B over every expert's rows of B give each expert's operands.
  pb2_noising_params qa{}, qb{};
  qa.device = p.device; qa.rows = p.m; qa.k = p.k; qa.r = p.r;
  qa.X = p.A; qa.EL = p.EAL; qa.E_rmajor = p.EAR_R_major; qa.E_kmajor = p.EBL_K_major;
  qa.XpE = p.ApEA; qa.proj = p.AxEBL_fp16; qa.proj_is_fp16 = 1;
  qa.host_signal_sync = all.host_signal_sync == &all ? nullptr : all.host_signal_sync;
  qb.device = p.device; qb.rows = E * p.n; qb.k = p.k; qb.r = p.r;
  qb.X = p.B; qb.EL = p.EBR; qb.E_rmajor = p.EBL_R_major; qb.E_kmajor = p.EAR_K_major;
  qb.XpE = p.BpEB; qb.proj = p.EARxBpEB_fp16; qb.proj_is_fp16 = 1;
  qb.host_signal_sync = qa.host_signal_sync;
  if (p.run_noising_a && p.run_noising_b) {
    if ((st = run_noising_both(qa, qb, s))) return st;
  } else if (p.run_noising_a) {
    if ((st = pb2_noise_A(&qa, stream))) return st;
  } else if (p.run_noising_b) {
    if ((st = pb2_noise_B(&qb, stream))) return st;
  }
  return run_grouped_kernel(p, gp->experts, E, gp->c_row_index, gp->c_rows, s);
}

namespace pb2 {
namespace {
template <int kKind>
int launch_fp8(const MainArgs& a, const ExpertTable<1>& x, int device, bool reduce, cudaStream_t s) {
  return reduce ? launch_variant<128, 1, true, false, false, BN, 1, kKind>(a, x, device, s)
                : launch_variant<128, 1, false, false, false, BN, 1, kKind>(a, x, device, s);
}
}  // namespace
}  // namespace pb2

extern "C" int pb2_mined_gemm_fp8(const pb2_fp8_gemm_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_mined_gemm_fp8");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_fp8_gemm_params& f = *pp;
  const bool reduce = !f.skip_reduction;
  if (f.format != PB2_FP8_E4M3 && f.format != PB2_FP8_E5M2) return PB2_ERR_UNSUPPORTED_CONFIG;
  if (f.r != 128) return PB2_ERR_UNSUPPORTED_CONFIG;
  // The same shape, pointer and buffer rules as the int8 mined GEMM.
  pb2_gemm_params q{};
  q.device = f.device;
  q.m = f.m; q.n = f.n; q.k = f.k; q.r = f.r;
  q.ApEA = const_cast<int8_t*>(static_cast<const int8_t*>(f.A));
  q.BpEB = const_cast<int8_t*>(static_cast<const int8_t*>(f.B));
  q.A_scales = f.A_scale;
  q.B_scales = f.B_scale;
  q.C = f.C;
  q.host_signal_header_pinned = f.host_signal_header_pinned;
  q.host_signal_sync = f.host_signal_sync;
  q.pow_target = f.pow_target;
  q.pow_key = f.pow_key;
  q.tile_size_m = BMC; q.tile_size_n = BN; q.tile_size_k = kTileK;
  q.cluster_size_m = q.cluster_size_n = 1;
  q.hits = f.hits; q.hit_capacity = f.hit_capacity;
  q.transcripts = f.transcripts; q.digests = f.digests;
  int st = check_main_args(q, reduce, false);
  if (st) return st;
  if ((st = set_device(f.device))) return st;
  MainArgs a;
  std::memset(&a, 0, sizeof(a));
  ExpertTable<1> x;
  std::memset(&x, 0, sizeof(x));
  if ((st = make_shared_args(a, q, 128, BN, false))) return st;
  if ((st = make_entry(x.ex[0], q.ApEA, nullptr, nullptr, f.A_scale, f.C, f.m, f.n, f.k, f.r, 128, false)))
    return st;
  x.count = 1;
  ExpertEntry& e = x.ex[0];
  e.sB = f.B_scale;
  e.sync = static_cast<SignalSync*>(f.host_signal_sync);
  e.header = static_cast<SignalHeader*>(f.host_signal_header_pinned);
  e.hits = f.hits;
  e.hit_cap = f.hits ? f.hit_capacity : 0;
  e.transcripts = f.transcripts;
  e.digests = f.digests;
  a.num_tiles = e.tiles_m * a.tiles_n;
  a.tpr = 2;
  a.scale_per_tensor = 1;
  a.sync = e.sync;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return f.format == PB2_FP8_E4M3 ? launch_fp8<1>(a, x, f.device, reduce, s) : launch_fp8<2>(a, x, f.device, reduce, s);
}
