/*
 * pearl_b200.h -- C ABI of the B200 (sm_100a) Pearl mining kernels.
 *
 * Plain pointers, sizes and a CUDA stream handle; no torch types.  Every
 * entry point is asynchronous on `stream` (a cudaStream_t passed as void*),
 * returns PB2_OK or a PB2_ERR_* code after validating its arguments, and
 * allocates nothing: the caller owns every input, output and scratch buffer,
 * exactly like the reference's pybind11 / TORCH_LIBRARY operators
 * (miner/pearl-gemm/csrc/gemm/pearl_gemm_api.cpp) whose argument lists the
 * parameter structs below mirror.  Device pointers must be on `device`.
 *
 * Matrix layouts are row-major and contiguous:
 *   A (m,k) int8, B (n,k) int8, EAL (m,r) int8, EBR (n,r) int8,
 *   EAR_R_major / EBL_R_major (k,r) int8, EAR_K_major / EBL_K_major (r,k) int8,
 *   *_fp16 (rows,r) IEEE half, AxEBL / EARxBpEB (rows,r) int32 or half,
 *   A_scales (m) / B_scales (n) float, C (m,n) bfloat16.
 */
#ifndef PEARL_B200_H_
#define PEARL_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define PB2_API __attribute__((visibility("default")))
#else
#define PB2_API
#endif

#define PB2_ABI_VERSION 1

/* Status codes. */
#define PB2_OK 0
#define PB2_ERR_INVALID_ARGUMENT 1 /* shape / alignment / missing tensor */
#define PB2_ERR_UNSUPPORTED_CONFIG 2 /* "No ... kernel found with given config" */
#define PB2_ERR_CUDA 3               /* a CUDA runtime call failed */
#define PB2_ERR_DEVICE_TIMEOUT 4     /* a bounded device-side wait ran out */
#define PB2_ERR_NO_DRIVER_ENTRY 5    /* cuTensorMapEncodeTiled unavailable */
#define PB2_ERR_SCRATCH_LIMIT 6      /* problem exceeds PB2_STATIC_SCRATCH_BYTES */

/* Sizes of the caller-owned signalling buffers.
 * Header: byte-compatible with the reference HostSignalHeader
 * (miner/pearl-gemm/csrc/gemm/host_signal_header.hpp:21-50), 640 bytes.
 * Sync: the reference HostSignalSync {int lock; int status} followed by
 * {uint32 hit_count; int32 error}; the caller zeroes it before each call. */
#define PB2_HOST_SIGNAL_HEADER_SIZE 640
#define PB2_HOST_SIGNAL_SYNC_SIZE 16
/* One entry of the optional device hit list:
 * {row_offset, col_offset, tile_m, tile_n, digest[8]} as uint32. */
#define PB2_HIT_WORDS 12

/* Replaces get_host_signal_header_size (pearl_gemm_api.cpp:48-50). */
PB2_API int64_t pb2_host_signal_header_size(void);
/* Replaces get_host_signal_sync_size (pearl_gemm_api.cpp:52-54). */
PB2_API int64_t pb2_host_signal_sync_size(void);
/* Human-readable text for a PB2_* status code (never NULL). */
PB2_API const char* pb2_status_string(int status);
/* Text of the last CUDA error seen by this library on the calling thread. */
PB2_API const char* pb2_last_cuda_error(void);
/* ABI version of the loaded library (PB2_ABI_VERSION). */
PB2_API int pb2_abi_version(void);

/* ------------------------------------------------------ bounded waits -----
 * No reference counterpart: the reference's kernels wait without limit (its
 * first-hit lock spins, pow_utils.hpp:267-269).  Every device-side wait of
 * these kernels (mbarrier phases, drains, cluster handshakes) gives up after
 * a budget of SM clock cycles, records PB2_ERR_DEVICE_TIMEOUT in the error
 * word of host_signal_sync and unwinds, so a stalled pipeline ends the
 * kernel with a status instead of holding the GPU.
 * pb2_set_wait_budget_cycles sets the budget that later launches of the
 * mined GEMM's main kernel (pb2_noisy_gemm, pb2_gemm) take, for the whole
 * process; cycles <= 0 restores the default (about one second).  Returns the
 * previous budget.  Launches already queued keep the budget they were
 * given.  The noising kernels always keep the default: their K-split
 * clusters read one another's shared memory until an exit handshake, which a
 * short budget must not cut.
 * pb2_wait_selftest launches one small kernel whose two warps wait on
 * mbarriers that nothing completes, with `budget_cycles`
 * (0 < budget_cycles <= the default): both waits run out, the error word
 * becomes PB2_ERR_DEVICE_TIMEOUT and the kernel returns. */
#define PB2_DEFAULT_WAIT_BUDGET_CYCLES 2000000000LL
PB2_API int64_t pb2_set_wait_budget_cycles(int64_t cycles);
PB2_API int pb2_wait_selftest(int device, int64_t budget_cycles, void* host_signal_sync, void* stream);

/* ----------------------------------------------------------- tensor_hash ---
 * Replaces tensor_hash (tensor_hash_api.hpp:45-120; kernels
 * merkle_tree_roots_kernel.hpp, compute_blake_mt_kernel.hpp,
 * reduce_roots_kernel.h): out = BLAKE3 keyed by `key` of the `len` bytes at
 * `data` zero-padded to whole 1 KiB chunks.  `roots` is caller scratch of at
 * least pb2_required_scratchpad_bytes(len, threads_per_block) bytes (one
 * 32-byte subtree root per group of threads_per_block chunks).  data must be
 * 16-byte aligned; key, out and roots 4-byte aligned; all on `device`.
 * threads_per_block in {128, 256, 512}; the reference's num_stages and
 * leaves_per_mt_block tuning knobs have no counterpart here. */
typedef struct pb2_tensor_hash_params {
  int device;
  const uint8_t* data;
  int64_t len;
  const uint8_t* key; /* 32 bytes */
  uint8_t* out;       /* 32 bytes */
  uint8_t* roots;     /* scratch */
  int64_t roots_bytes;
  int threads_per_block;
} pb2_tensor_hash_params;
PB2_API int pb2_tensor_hash(const pb2_tensor_hash_params* p, void* stream);
/* Replaces get_required_scratchpad_bytes (tensor_hash_api.hpp:37-43). */
PB2_API int64_t pb2_required_scratchpad_bytes(int64_t matrix_bytes, int threads_per_block);

/* --------------------------------------------------------- merkle layers ---
 * Replaces building pearl_mining.MerkleTree on the host for a hit's proof
 * (pearl-blake3/src/merkle.rs:43-81, called by miner_base
 * matrix_merkle_tree.py:26 and block_submission.py:25-26, zk-pow
 * src/ffi/mine.rs:385): every layer of the keyed BLAKE3 tree over the `len`
 * bytes at `data` zero-padded to whole 1 KiB chunks, leaves first, 32 bytes
 * per node, layers back to back.  Layer 0 has one node per chunk; while a
 * layer has more than two nodes the next has ceil(n / 2) (neighbours paired,
 * an odd node carried up); a two-node layer is followed by the one-node root
 * layer; a single chunk is its own root.  The last node is the tensor_hash of
 * the same bytes.  `nodes` holds at least pb2_merkle_nodes(len) * 32 bytes.
 * data 16-byte aligned; key and nodes 4-byte aligned; all on `device`. */
typedef struct pb2_merkle_params {
  int device;
  const uint8_t* data;
  int64_t len;
  const uint8_t* key; /* 32 bytes */
  uint8_t* nodes;
  int64_t nodes_bytes;
} pb2_merkle_params;
PB2_API int pb2_merkle_layers(const pb2_merkle_params* p, void* stream);
/* Total node count of all layers for `len` bytes (0 when len <= 0). */
PB2_API int64_t pb2_merkle_nodes(int64_t len);

/* ------------------------------------- commitment_hash_from_merkle_roots ---
 * Replaces commitment_hash_from_merkle_roots (tensor_hash_api.hpp:124-212,
 * commitment_hash_from_merkle_roots_kernel.hpp): the noise seeds
 *   B_commitment_hash = BLAKE3(key || B_root'),
 *   A_commitment_hash = BLAKE3(B_commitment_hash || A_root'),
 * where with `salted` each root is first bound to its matrix dimension
 * (V3 seeds) and, when routing_root / offsets_hash are given (MoE),
 * A_root' = BLAKE3(A_root || BLAKE3(routing_root || offsets_hash)).
 * All buffers are 32 bytes on `device`, 4-byte aligned. */
typedef struct pb2_commitment_params {
  int device;
  const uint8_t* A_merkle_root;
  const uint8_t* B_merkle_root;
  const uint8_t* key;
  uint8_t* A_commitment_hash;
  uint8_t* B_commitment_hash;
  const uint8_t* routing_root; /* optional, with offsets_hash */
  const uint8_t* offsets_hash;
  int salted;
  uint32_t salted_dim_a, salted_dim_b;
} pb2_commitment_params;
PB2_API int pb2_commitment_hash_from_merkle_roots(const pb2_commitment_params* p, void* stream);

/* ---------------------------------------------------- build_routing_data ---
 * Replaces build_routing_data (miner/pearl-gemm/csrc/moe/build_routing_data.cu:
 * 40-166): for the (num_tokens, top_k) int32 expert ids, slot_indices = flat
 * slot indices stably sorted by expert id (8-bit ids, num_experts <= 256),
 * routing_data = slot_indices / top_k, routing_offsets[e] = number of slots
 * with expert id <= e.  scratchpad: at least
 * pb2_build_routing_data_scratchpad_bytes(num_tokens * top_k) bytes, 4-byte
 * aligned. */
typedef struct pb2_routing_params {
  int device;
  const int32_t* topk_ids; /* (num_tokens, top_k) */
  int64_t num_tokens, top_k;
  int32_t* routing_data;    /* (num_tokens * top_k) */
  int32_t* slot_indices;    /* (num_tokens * top_k) */
  int32_t* routing_offsets; /* (num_experts) */
  int64_t num_experts;
  void* scratchpad;
  int64_t scratchpad_bytes;
} pb2_routing_params;
PB2_API int pb2_build_routing_data(const pb2_routing_params* p, void* stream);
/* Replaces get_build_routing_data_scratchpad_bytes (build_routing_data.cu:113-125). */
PB2_API int64_t pb2_build_routing_data_scratchpad_bytes(int64_t numel);

/* -------------------------------------------------------------- quantize ---
 * Replaces pearl_gemm.quantization.quantize (hadamard.py:530-611), the
 * activation quantization the mining layer runs before the GEMM
 * (quantization_operators.py:72-100): per row of x (m, n) bf16 or fp16,
 * optional block Walsh-Hadamard transform of width block_size (0 = none; else
 * a power of two in [8, 256] dividing n), times smooth (1 x n, or m x n when
 * smooth_per_row; may be NULL), then xq = rint(v * inv) clamped to +-max_val
 * with inv = max_val * rcp.approx.ftz(amax + 1e-30), and scales[row] =
 * amax * fl(1 / max_val) (hadamard.py:443-466, the same float32 steps).
 * x and smooth 16-byte aligned, xq 8-byte aligned.
 * Narrower than the reference: n % 8 == 0 (16-byte row vectors; model
 * widths always are) and block_size >= 8.  The reference's layout puts
 * gcd(n, 8) elements in a thread, and for a block narrower than that its
 * per-block negation index k / vecsize is zero (hadamard.py:505-511), so
 * widths 2 and 4 have no well-defined reference result to match; both
 * cases return PB2_ERR_UNSUPPORTED_CONFIG. */
typedef struct pb2_quant_params {
  int device;
  const void* x;
  int x_is_fp16; /* 0: bfloat16 */
  int64_t m, n;
  const float* smooth;
  int smooth_per_row;
  int8_t* xq;
  float* scales; /* (m) */
  int max_val;   /* 63 (7-bit) or 127 (8-bit) */
  int block_size;
} pb2_quant_params;
PB2_API int pb2_quantize(const pb2_quant_params* p, void* stream);
/* Test aid, no reference counterpart: out[i] = rcp.approx.ftz.f32(in[i]) on
 * `device`, the approximate reciprocal pb2_quantize takes as the reference's
 * kernel does (cute.arch.rcp_approx).  PTX bounds its error (1 ulp) but does
 * not fix its last bit, so a CPU restatement of the quantizer reads it from
 * the device.  in and out hold n floats on `device`. */
PB2_API int pb2_rcp_approx_f32(int device, const float* in, float* out, int64_t n, void* stream);

/* ---------------------------------------------------------- scatter_rows ---
 * dst[indices[i]] = src[i] for i < rows, rows of row_bytes bytes (a multiple
 * of 16; src, dst 16-byte aligned; indices int32).  Replaces the per-expert
 * row scatter of the mined MoE layer, cache_flat[expert_slot_indices] =
 * expert_output (miner/vllm-miner/src/vllm_miner/pearl_moe_experts.py:347),
 * which torch runs as an index_put.  Indices outside [0, dst_rows) are
 * skipped; duplicated indices leave one of their rows (unspecified which). */
typedef struct pb2_scatter_params {
  int device;
  const void* src;      /* (rows, row_bytes) */
  void* dst;            /* (dst_rows, row_bytes) */
  const int32_t* indices; /* (rows) */
  int64_t rows, dst_rows, row_bytes;
} pb2_scatter_params;
PB2_API int pb2_scatter_rows(const pb2_scatter_params* p, void* stream);

/* ------------------------------------------------------------- noise_gen ---
 * Replaces noise_gen (pearl_gemm_api.cpp:168-298; kernel
 * noise_generation_kernel.h:88-758).  Any output may be NULL (not produced).
 * Sparse outputs are fully written (zeros included).  key_a / key_b are
 * 32-byte device buffers; key_a is required when any A-side output is
 * requested, key_b for B-side outputs.  aux_buffer (aux_words uint32,
 * aux_words % 4 == 0) is zeroed when given. */
typedef struct pb2_noise_gen_params {
  int device;
  int64_t m, n, k, r;
  int8_t* EAL;          /* (m,r)  */
  void* EAL_fp16;       /* (m,r) half, value * kEALScaleFactorDenoise (-1) */
  int8_t* EAR_R_major;  /* (k,r)  */
  int8_t* EAR_K_major;  /* (r,k)  */
  int8_t* EBL_R_major;  /* (k,r)  */
  int8_t* EBL_K_major;  /* (r,k)  */
  int8_t* EBR;          /* (n,r)  */
  void* EBR_fp16;       /* (n,r) half, value * kEBRScaleFactorDenoise (-4) */
  const uint8_t* key_a; /* 32 bytes */
  const uint8_t* key_b; /* 32 bytes */
  uint32_t* aux_buffer;
  int64_t aux_words;
} pb2_noise_gen_params;
PB2_API int pb2_noise_gen(const pb2_noise_gen_params* p, void* stream);

/* ------------------------------------------------------- noise_A / noise_B -
 * noise_A replaces pearl_gemm_api.cpp:300-398:
 *   ApEA = A + EAL . EAR^T                (EAR given as (k,r) R-major)
 *   AxEBL = A . EBL^T, EBL given as (r,k) K-major; int32 exact, or half
 *   scaled by 2^-14 when out_is_fp16.
 * noise_B replaces pearl_gemm_api.cpp:400-500:
 *   BpEB = B + EBR . EBL^T               (EBL given as (k,r) R-major)
 *   EARxBpEB = BpEB . EAR^T, EAR given as (r,k) K-major; int32 or half * 2^-12.
 * The generic form below serves both: X = A or B, EL = EAL or EBR,
 * E_rmajor = EAR_R_major or EBL_R_major, E_kmajor = EBL_K_major or
 * EAR_K_major.  int32 outputs are ACCUMULATED (atomic adds; zero them first,
 * as the reference requires for its split-K path); half outputs are written.
 * For noise_B the projection uses the noised operand XpE. */
typedef struct pb2_noising_params {
  int device;
  int64_t rows, k, r;
  const int8_t* X;        /* (rows,k) */
  const int8_t* EL;       /* (rows,r) */
  const int8_t* E_rmajor; /* (k,r)    */
  const int8_t* E_kmajor; /* (r,k)    */
  int8_t* XpE;            /* (rows,k) out */
  void* proj;             /* (rows,r) out, int32 or half */
  int proj_is_fp16;
  int k_blocks_per_split; /* <0: heuristic; 0: no split; >0: k-blocks of 128 per CTA */
  void* host_signal_sync; /* optional: receives PB2_ERR_DEVICE_TIMEOUT in its error word */
} pb2_noising_params;
PB2_API int pb2_noise_A(const pb2_noising_params* p, void* stream);
PB2_API int pb2_noise_B(const pb2_noising_params* p, void* stream);
/* noise_A(a) and noise_B(b) of one mined GEMM, exactly as the two calls
 * above (same outputs, same validation), in one launch when both
 * projections are half precision with the same r and k, else as two.  No
 * reference counterpart of its own: it is the noising step that
 * noisy_gemm(run_noising_A, run_noising_B) performs before its GEMM
 * (pearl_gemm_api.cpp:879-892), exposed so a caller can time it apart. */
PB2_API int pb2_noise_AB(const pb2_noising_params* a, const pb2_noising_params* b, void* stream);

/* ----------------------------------------------------- denoise_converter ---
 * Replaces denoise_converter (pearl_gemm_api.cpp:114-166): int32 -> half
 * with scale 2^-12 (EARxBpEB) and 2^-14 (AxEBL).  Either pair may be NULL. */
typedef struct pb2_denoise_converter_params {
  int device;
  int64_t m, n, r;
  const int32_t* EARxBpEB_in; /* (n,r) */
  const int32_t* AxEBL_in;    /* (m,r) */
  void* EARxBpEB_out;         /* (n,r) half */
  void* AxEBL_out;            /* (m,r) half */
} pb2_denoise_converter_params;
PB2_API int pb2_denoise_converter(const pb2_denoise_converter_params* p, void* stream);

/* ------------------------------------------------------ noisy_gemm / gemm ---
 * Replaces noisy_gemm (pearl_gemm_api.cpp:618-936) and gemm (:502-616).
 * The main kernel computes, per 128 x 256 output tile,
 *   S = ApEA . BpEB^T (int32, tcgen05 int8 MMA, accumulator in TMEM),
 * folds the protocol transcript of every 2 x 64 hash tile every r steps of k,
 * hashes it with keyed BLAKE3 (key = pow_key) and compares with pow_target,
 * then (unless skip_denoising)
 *   C = bf16(A_scales[m] * B_scales[n] *
 *            (S + EAL_fp16 . EARxBpEB_fp16^T * 2^12 + AxEBL_fp16 . EBR_fp16^T * 2^12)).
 * run_noising_a / run_noising_b run noise_A / noise_B first (from A, EAL,
 * EAR_R_major, EBL_K_major / B, EBR, EAR_K_major, EBL_R_major); the int32
 * denoise factors, when given, are produced there and converted to half.
 * Hits: the first in-bounds hit writes the pinned host header and sets
 * sync->status (no spinning); every hit is appended to the optional device
 * hit list.  The optional debug outputs (transcripts, digests: one slot per
 * protocol hash tile, index (row/16*8 + row%16) * (n/64) + col/256*4 + (col%256)/2;
 * inner_hash_counter: one count per hash-tile fold) need m % 16 == 0 and
 * n % 256 == 0. */
typedef struct pb2_gemm_params {
  int device;
  int64_t m, n, k, r;
  /* inputs of the optional noising stage */
  const int8_t* A;
  const int8_t* B;
  const int8_t* EAL;
  const int8_t* EBR;
  const int8_t* EAR_R_major;
  const int8_t* EBL_R_major;
  const int8_t* EAR_K_major;
  const int8_t* EBL_K_major;
  int32_t* AxEBL_int32;    /* optional */
  int32_t* EARxBpEB_int32; /* optional */
  /* main kernel operands */
  int8_t* ApEA;            /* (m,k) */
  int8_t* BpEB;            /* (n,k) */
  const void* EAL_fp16;    /* (m,r) half */
  const void* EBR_fp16;    /* (n,r) half */
  void* AxEBL_fp16;        /* (m,r) half */
  void* EARxBpEB_fp16;     /* (n,r) half */
  const float* A_scales;   /* (m) */
  const float* B_scales;   /* (n) */
  void* C;                 /* (m,n) bf16 */
  void* host_signal_header_pinned; /* PB2_HOST_SIGNAL_HEADER_SIZE bytes, host pinned */
  void* host_signal_sync;          /* PB2_HOST_SIGNAL_SYNC_SIZE bytes, device */
  const uint32_t* pow_target;      /* 8 words, little-endian word order */
  const uint32_t* pow_key;         /* 8 words */
  /* tile / schedule knobs (reference names) */
  int tile_size_m, tile_size_n, tile_size_k;
  int cluster_size_m, cluster_size_n;
  int pipeline_stages; /* <= 0: default */
  int swizzle;         /* <= 0: heuristic; raster group size in tiles */
  int swizzle_n_maj;
  int run_noising_a, run_noising_b;
  int k_blocks_per_split_noising_a, k_blocks_per_split_noising_b;
  int skip_reduction, skip_denoising;
  /* B200 extensions (all optional) */
  uint64_t* inner_hash_counter;
  int enable_debug;
  uint32_t* hits;        /* hit_capacity * PB2_HIT_WORDS words */
  int64_t hit_capacity;
  uint32_t* transcripts; /* (m/2)*(n/64) * 16 words */
  uint32_t* digests;     /* (m/2)*(n/64) * 8 words  */
  /* pb2_gemm only (optional): scratch for a K split of a GEMM with too few
   * tiles to fill the SMs (a decode batch), pb2_gemm_workspace_bytes() bytes,
   * 16-byte aligned, on `device`.  Null or smaller: no split. */
  int32_t* workspace;
  int64_t workspace_bytes;
} pb2_gemm_params;
PB2_API int pb2_noisy_gemm(const pb2_gemm_params* p, void* stream);
/* Plain scaled GEMM: C = bf16(A_scales * (A . B^T) * B_scales), reading the
 * operands from p->ApEA / p->BpEB (the reference passes A and B there).
 * No reference counterpart for the workspace: when few 256 x 256 tiles
 * cover C (m a decode batch), K is cut into equal ranges, every (tile, range)
 * runs on its own SM pair and writes its exact int32 partial to the
 * workspace, and a second kernel sums the ranges and applies the scales --
 * the same C, bit for bit, as without the split. */
PB2_API int pb2_gemm(const pb2_gemm_params* p, void* stream);
/* Bytes of workspace pb2_gemm would use for this shape on `device` (0: it
 * would not split K). */
PB2_API int64_t pb2_gemm_workspace_bytes(int device, int64_t m, int64_t n, int64_t k);

/* ------------------------------------------------------ FP8 mined GEMM ---
 * No reference counterpart: the protocol defines mined GEMMs of 7-bit
 * integers only (zk-pow/src/api/proof.rs:23-25), and the reference's only
 * FP8 GEMM is the un-mined MoE GEMM2 (pearl_moe_experts.py:377-434).  This
 * is the same mined GEMM on FP8 operands (both E4M3 or both E5M2) with
 * per-tensor scales:
 *   S = A . B^T accumulated in f32 on the tensor cores (kind::f8f6f4),
 * the transcript of every 2 x 64 hash tile folded from the f32 accumulator
 * BIT PATTERNS every r = 128 steps of k exactly as the int8 path folds its
 * int32 words, keyed BLAKE3 (pow_key) and the target compare, hits as for
 * pb2_noisy_gemm, and C = bf16(S * A_scale[0] * B_scale[0]).  No noise and
 * no denoise terms.  The f32 accumulation order inside the tensor core is
 * not specified, so the transcript is reproducible off the device only
 * where every partial sum is exact (integer-valued operands with
 * |partial sums| < 2^24).  Same shape rules as pb2_noisy_gemm (k % 128 == 0,
 * n % 8 == 0, dumps need m % 16 == 0 and n % 256 == 0); A, B, C 16-byte
 * aligned; the scales are one float each on `device`. */
#define PB2_FP8_E4M3 0
#define PB2_FP8_E5M2 1
typedef struct pb2_fp8_gemm_params {
  int device;
  int64_t m, n, k, r;    /* r: transcript period, 128 */
  const void* A;         /* (m,k) FP8 */
  const void* B;         /* (n,k) FP8 */
  int format;            /* PB2_FP8_E4M3 or PB2_FP8_E5M2 (both operands) */
  const float* A_scale;  /* 1 float */
  const float* B_scale;  /* 1 float */
  void* C;               /* (m,n) bf16 */
  void* host_signal_header_pinned;
  void* host_signal_sync;
  const uint32_t* pow_target;
  const uint32_t* pow_key;
  int skip_reduction;
  uint32_t* hits;
  int64_t hit_capacity;
  uint32_t* transcripts;
  uint32_t* digests;
} pb2_fp8_gemm_params;
PB2_API int pb2_mined_gemm_fp8(const pb2_fp8_gemm_params* p, void* stream);

/* ---------------------------------------------------- grouped noisy_gemm ---
 * Replaces the per-expert loop of the mined MoE GEMM1
 * (miner/vllm-miner/src/vllm_miner/pearl_moe_experts.py:304-343, each pass a
 * moe_gemm_operators.py:259-329 noisy_gemm with run_noising_A/B): the
 * experts' mined GEMMs in one noising launch and one persistent main launch
 * per 16 experts, with the same results as one pb2_noisy_gemm per expert.
 * `shared` holds the stacked problem: m = all experts' rows, A-side arrays
 * (A, EAL, ApEA, EAL_fp16, AxEBL_fp16, A_scales, C) with those m rows in
 * expert order, B-side arrays (B, EBR, BpEB, EBR_fp16, EARxBpEB_fp16,
 * B_scales) with n rows per expert (expert e at rows [e n, e n + n)), the
 * shared K-side factors, r, k, pow_target, pow_key and the tile knobs; its
 * host_signal_*, hits, transcripts and digests are not used.  Expert e
 * takes rows [a_row0, a_row0 + m) of the A-side arrays (a_row0 = the sum of
 * the earlier experts' m; m may be 0) and reports its hits through its own
 * sync word, pinned header and optional hit list and debug dumps, indexed
 * as for a pb2_noisy_gemm of its m rows.  A device timeout is recorded in
 * the first non-empty expert's sync word.  Half-precision projections only
 * (AxEBL_int32 / EARxBpEB_int32 NULL); skip_reduction, skip_denoising and
 * enable_debug must be 0. */
typedef struct pb2_expert_gemm {
  int64_t m;
  int64_t a_row0;
  void* host_signal_header_pinned; /* optional */
  void* host_signal_sync;          /* required when m > 0 */
  uint32_t* hits;                  /* optional, hit_capacity * PB2_HIT_WORDS words */
  int64_t hit_capacity;
  uint32_t* transcripts;           /* optional, (m/2)*(n/64) * 16 words */
  uint32_t* digests;               /* optional, (m/2)*(n/64) * 8 words */
} pb2_expert_gemm;
typedef struct pb2_grouped_gemm_params {
  pb2_gemm_params shared;
  int64_t num_experts;
  const pb2_expert_gemm* experts; /* host array of num_experts entries */
  /* Optional row map (no reference counterpart): row r of the stacked C is
   * written to row c_row_index[r] of shared.C, a destination of c_rows >= m
   * rows (rows outside it skipped) -- the slot-order write-back that follows
   * the reference's loop (pearl_moe_experts.py:347, cache_flat[idx] = out)
   * fused into the epilogue.  int32, device, m entries. */
  const int32_t* c_row_index;
  int64_t c_rows;
} pb2_grouped_gemm_params;
PB2_API int pb2_noisy_gemm_grouped(const pb2_grouped_gemm_params* p, void* stream);

/* ------------------------------------------- noisy_gemm, static scratch ---
 * No counterpart in the reference.  The same mined GEMM as pb2_noisy_gemm,
 * for callers that cannot allocate device memory: a host that only reaches
 * this library through its C ABI and has no device allocator, or a process
 * whose HBM is owned by another allocator (an inference server's memory pool
 * takes most of it at start-up, so a cudaMalloc can fail, and a cudaFree
 * stalls the whole device).  The exact int32 noising projections, which
 * pb2_noisy_gemm reads from the caller's AxEBL_int32 / EARxBpEB_int32, live
 * in a fixed array inside the library instead; p->AxEBL_int32 and
 * p->EARxBpEB_int32 must be NULL.  Every other argument, and every result,
 * is as for pb2_noisy_gemm (the caller still passes all inputs and outputs).
 *   Limit: (m if run_noising_a) * r + (n if run_noising_b) * r int32 words
 *   must fit in PB2_STATIC_SCRATCH_BYTES (8 MiB: m + n <= 16384 at r = 128);
 *   larger problems return PB2_ERR_SCRATCH_LIMIT before any work is queued.
 * Each GPU that loads the library holds the array until the process exits.
 * The first call on a device looks up the array's device address (with that
 * device current) and caches it; make that first call before any stream
 * capture.  No call allocates device or host memory.  All calls on a device
 * share the array, which keeps the last call's contents: each call clears
 * the words it uses on `stream` first, and calls that overlap on the GPU
 * (unordered streams) race on it. */
#define PB2_STATIC_SCRATCH_BYTES (8 * 1024 * 1024)
PB2_API int pb2_noisy_gemm_static_scratch(const pb2_gemm_params* p, void* stream);

/* -------------------------------------------------------------- inner_hash -
 * Replaces inner_hash (pearl_gemm_api.cpp:939-970, inner_hash_kernel.cu:11-58):
 * out[0] = the XOR of in[0..n) added up `iterations` times (mod 2^32), with
 * n in {64,96,128,192,256} and iterations in {1, 100000}. */
PB2_API int pb2_inner_hash(int device, const uint32_t* in, int64_t n, uint32_t* out, int64_t iterations,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PEARL_B200_H_ */
