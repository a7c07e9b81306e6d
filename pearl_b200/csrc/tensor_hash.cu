// tensor_hash.cu -- the commitment inputs of a mined GEMM on sm_100a.
//
// tensor_hash: keyed BLAKE3 of a byte tensor zero-padded to whole 1 KiB
// chunks (pearl-blake3/src/merkle.rs:15-27; the reference's GPU version is
// miner/pearl-gemm/csrc/tensor_hash/tensor_hash_api.hpp:37-120).  BLAKE3's
// tree is left-heavy: every aligned power-of-two run of chunks is a complete
// subtree, and the tree above such runs is obtained by merging neighbours
// pairwise level by level, an odd node carried up unchanged.  So one CTA
// hashes a group of `threads_per_block` chunks (one chunk per thread, sixteen
// chained compressions), folds the group's chaining values in shared memory
// into the group's subtree root, and writes it to the caller's scratch; a
// single CTA then folds the group roots the same way.  With one group the
// first kernel applies the ROOT flag itself.  The scratch size is the
// reference's (get_required_scratchpad_bytes, tensor_hash_api.hpp:37-43).
//
// Work per 64 MiB operand: 65,536 chunks x 16 compressions (~700 integer
// instructions each): about 20 us of integer issue on 148 SMs against 10 us
// of HBM reads, so the kernel is issue-bound and every load is a single
// 16-byte read-only load of the thread's own chunk (the 128-byte line it
// opens serves the next block from L1).
//
// commitment_hash_from_merkle_roots: the noise-seed chain from the two roots
// (commitment_hash_from_merkle_roots_kernel.hpp; protocol
// zk-pow/src/api/proof_utils.rs:361-372, api/seed.rs:20-58, MoE fold
// proof_utils.rs:34-45).  One thread: a handful of single-block compressions.
#include "pb2_common.cuh"

namespace pb2 {
namespace {

constexpr int kChunkBytes = 1024;

// The BLAKE3 IV (the unkeyed hash's initial chaining value).
__device__ __forceinline__ void b3_iv(uint32_t* iv) {
  iv[0] = kB3IV0; iv[1] = kB3IV1; iv[2] = kB3IV2; iv[3] = kB3IV3;
  iv[4] = 0x510E527Fu; iv[5] = 0x9B05688Cu; iv[6] = 0x1F83D9ABu; iv[7] = 0x5BE0CD19u;
}

struct TensorHashArgs {
  const uint8_t* data;
  uint64_t len;
  uint64_t chunks;
  uint32_t num_groups;
  const uint32_t* key;
  uint32_t* roots;
  uint32_t* out;
};

// Message words of 64-byte block `b` of chunk `c` (zero past the data).
__device__ __forceinline__ void load_block(const TensorHashArgs& a, uint64_t c, int b, uint32_t* m) {
  const uint64_t off = c * kChunkBytes + uint64_t(b) * 64;
  if (off + 64 <= a.len) {
    const uint4* p = reinterpret_cast<const uint4*>(a.data + off);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 q = __ldg(p + j);
      m[4 * j] = q.x;
      m[4 * j + 1] = q.y;
      m[4 * j + 2] = q.z;
      m[4 * j + 3] = q.w;
    }
  } else {  // the ragged end of the data (unrolled: m stays in registers)
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t idx = off + 4 * w + i;
        if (idx < a.len) word |= uint32_t(a.data[idx]) << (8 * i);
      }
      m[w] = word;
    }
  }
}

// Chaining value of chunk c (its hash when `root`: the whole input is c).
__device__ void chunk_cv(const TensorHashArgs& a, const uint32_t* key, uint64_t c, bool root,
                         uint32_t* cv) {
#pragma unroll
  for (int i = 0; i < 8; ++i) cv[i] = key[i];
  // Block b + 1 is loaded before block b is compressed, so its latency hides
  // behind the compression (a warp per SM sub-partition is all a 64 MiB
  // tensor offers: one thread per chunk, sixteen dependent compressions).
  uint32_t m[16];
  load_block(a, c, 0, m);
#pragma unroll 1
  for (int b = 0; b < kChunkBytes / 64; ++b) {
    uint32_t mn[16];
    if (b + 1 < kChunkBytes / 64) load_block(a, c, b + 1, mn);
    uint32_t flags = kB3Keyed;
    if (b == 0) flags |= kB3ChunkStart;
    if (b == kChunkBytes / 64 - 1) flags |= kB3ChunkEnd | (root ? kB3Root : 0u);
    uint32_t next[8];
    b3_compress8_at(cv, m, c, 64, flags, next);
#pragma unroll
    for (int i = 0; i < 8; ++i) cv[i] = next[i];
    if (b + 1 < kChunkBytes / 64) {
#pragma unroll
      for (int i = 0; i < 16; ++i) m[i] = mn[i];
    }
  }
}

__device__ __forceinline__ void parent_cv(const uint32_t* key, const uint32_t* left, const uint32_t* right,
                                          bool root, uint32_t* out) {
  uint32_t m[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m[i] = left[i];
    m[8 + i] = right[i];
  }
  b3_compress8_at(key, m, 0, 64, kB3Parent | kB3Keyed | (root ? kB3Root : 0u), out);
}

template <int TPB>
__global__ void __launch_bounds__(TPB) chunk_group_kernel(const TensorHashArgs a) {
  __shared__ uint32_t cvs[TPB][9];  // 9-word rows: conflict-free column access
  __shared__ uint32_t key[8];
  const int t = threadIdx.x;
  const uint64_t first = uint64_t(blockIdx.x) * TPB;
  const int n = int(a.chunks - first < uint64_t(TPB) ? a.chunks - first : uint64_t(TPB));
  const bool single = a.num_groups == 1;  // this group is the whole tree
  if (t < 8) key[t] = a.key[t];
  __syncthreads();
  if (t < n) {
    uint32_t cv[8];
    chunk_cv(a, key, first + t, single && a.chunks == 1, cv);
#pragma unroll
    for (int i = 0; i < 8; ++i) cvs[t][i] = cv[i];
  }
  __syncthreads();
  for (int cnt = n; cnt > 1;) {
    const int pairs = cnt / 2;
    uint32_t out[8];
    if (t < pairs) parent_cv(key, cvs[2 * t], cvs[2 * t + 1], single && cnt == 2, out);
    __syncthreads();
    if (t < pairs) {
#pragma unroll
      for (int i = 0; i < 8; ++i) cvs[t][i] = out[i];
    }
    if ((cnt & 1) && t < 8) cvs[pairs][t] = cvs[cnt - 1][t];  // odd node carried up
    __syncthreads();
    cnt = pairs + (cnt & 1);
  }
  if (t < 8) {
    if (single)
      a.out[t] = cvs[0][t];
    else
      a.roots[uint64_t(blockIdx.x) * 8 + t] = cvs[0][t];
  }
}

// Folds num_groups >= 2 group roots (in place in the scratch) to the hash.
__global__ void __launch_bounds__(1024) root_fold_kernel(const TensorHashArgs a) {
  __shared__ uint32_t key[8];
  const uint32_t t = threadIdx.x;
  if (t < 8) key[t] = a.key[t];
  __syncthreads();
  uint32_t* nodes = a.roots;
  for (uint32_t cnt = a.num_groups; cnt > 1;) {
    const uint32_t pairs = cnt / 2;
    // Pass `base` writes nodes [base, base + 1024) and later passes read from
    // 2 * (base + 1024) on, so the level can be folded in place.
    for (uint32_t base = 0; base < pairs; base += blockDim.x) {
      const uint32_t i = base + t;
      uint32_t out[8];
      if (i < pairs) parent_cv(key, nodes + 16ull * i, nodes + 16ull * i + 8, cnt == 2, out);
      __syncthreads();
      if (i < pairs) {
#pragma unroll
        for (int w = 0; w < 8; ++w) nodes[8ull * i + w] = out[w];
      }
      __syncthreads();
    }
    if (cnt & 1) {
      if (t < 8) nodes[8ull * pairs + t] = nodes[8ull * (cnt - 1) + t];
      __syncthreads();
    }
    cnt = pairs + (cnt & 1);
  }
  if (t < 8) a.out[t] = nodes[t];
}

// ------------------------------------------------------------ merkle layers
// Every layer of the tree tensor_hash folds, kept for a proof of a hit's rows
// (pearl-blake3/src/merkle.rs:43-81 over the zero-padded tensor): layer 0
// holds one CV per chunk; while a layer has more than two nodes the next one
// pairs neighbours (an odd node carried up unchanged); a two-node layer is
// followed by the root (ROOT flag).  A single chunk is its own root.  One
// 128-thread CTA per group of 128 aligned chunks writes layers 0-7 of its
// group (all of them when the group is the whole tree); one CTA then builds
// the layers above 7 from the group nodes.
constexpr int kMerkleGroup = 128;
constexpr int kMerkleGroupLevels = 7;  // log2(kMerkleGroup)
constexpr int kMerkleMaxLayers = 64;

struct MerkleArgs {
  TensorHashArgs h;  // data, len, chunks, num_groups (of kMerkleGroup chunks), key
  uint32_t* nodes;   // 8 words per node, layers back to back
  uint64_t off[kMerkleMaxLayers];
  int layers;
};

__global__ void __launch_bounds__(kMerkleGroup) merkle_group_kernel(const MerkleArgs a) {
  __shared__ uint32_t cvs[kMerkleGroup][9];
  __shared__ uint32_t key[8];
  const int t = threadIdx.x;
  const uint64_t first = uint64_t(blockIdx.x) * kMerkleGroup;
  const int n = int(a.h.chunks - first < uint64_t(kMerkleGroup) ? a.h.chunks - first : uint64_t(kMerkleGroup));
  const bool single = a.h.num_groups == 1;
  if (t < 8) key[t] = a.h.key[t];
  __syncthreads();
  if (t < n) {
    uint32_t cv[8];
    chunk_cv(a.h, key, first + t, a.h.chunks == 1, cv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      cvs[t][i] = cv[i];
      a.nodes[(a.off[0] + first + t) * 8 + i] = cv[i];
    }
  }
  __syncthreads();
  // A group that is the whole tree folds to the root; otherwise every group
  // folds to its layer-7 node, a short last group carrying its last node up.
  const int top = single ? a.layers - 1 : kMerkleGroupLevels;
  int cnt = n;
  for (int l = 1; l <= top; ++l) {
    const int pairs = cnt / 2;
    uint32_t out[8];
    if (t < pairs) parent_cv(key, cvs[2 * t], cvs[2 * t + 1], single && cnt == 2, out);
    __syncthreads();
    if (t < pairs) {
#pragma unroll
      for (int i = 0; i < 8; ++i) cvs[t][i] = out[i];
    }
    if ((cnt & 1) && t < 8) cvs[pairs][t] = cvs[cnt - 1][t];
    __syncthreads();
    cnt = pairs + (cnt & 1);
    uint32_t* dst = a.nodes + (a.off[l] + (first >> l)) * 8;
    for (int e = t; e < cnt * 8; e += kMerkleGroup) dst[e] = cvs[e >> 3][e & 7];
  }
}

__global__ void __launch_bounds__(1024) merkle_top_kernel(const MerkleArgs a) {
  __shared__ uint32_t key[8];
  const uint32_t t = threadIdx.x;
  if (t < 8) key[t] = a.h.key[t];
  __syncthreads();
  uint64_t cnt = a.h.num_groups;
  for (int l = kMerkleGroupLevels + 1; l < a.layers; ++l) {
    const uint32_t* prev = a.nodes + a.off[l - 1] * 8;
    uint32_t* next = a.nodes + a.off[l] * 8;
    const uint64_t pairs = cnt / 2;
    for (uint64_t i = t; i < pairs; i += blockDim.x) {
      uint32_t out[8];
      parent_cv(key, prev + 16 * i, prev + 16 * i + 8, cnt == 2, out);
#pragma unroll
      for (int w = 0; w < 8; ++w) next[8 * i + w] = out[w];
    }
    if ((cnt & 1) && t < 8) next[8 * pairs + t] = prev[8 * (cnt - 1) + t];
    __syncthreads();
    cnt = pairs + (cnt & 1);
  }
}

// ---------------------------------------------------------------- commitment
struct CommitArgs {
  const uint32_t* root_a;
  const uint32_t* root_b;
  const uint32_t* key;
  uint32_t* out_a;
  uint32_t* out_b;
  const uint32_t* routing_root;  // MoE: both or neither
  const uint32_t* offsets_hash;
  int salted;
  uint32_t dim_a, dim_b;
};

// Unkeyed BLAKE3 of one 64-byte message (left || right): a single chunk of
// one block.
__device__ void hash64(const uint32_t* left, const uint32_t* right, uint32_t* out) {
  uint32_t m[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m[i] = left[i];
    m[8 + i] = right[i];
  }
  uint32_t iv[8];
  b3_iv(iv);
  b3_compress8_at(iv, m, 0, 64, kB3ChunkStart | kB3ChunkEnd | kB3Root, out);
}

// V3 domain-separation salt: unkeyed BLAKE3 of "pearl/cert-v3/noise-seed/A"
// or ".../B" (api/seed.rs:31-39), hashed here rather than stored.
__device__ void seed_salt(bool b_side, uint32_t* out) {
  const char kText[] = "pearl/cert-v3/noise-seed/A";
  constexpr int kLen = sizeof(kText) - 1;
  uint32_t m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = 0;
  for (int i = 0; i < kLen; ++i) {
    const uint32_t ch = (i == kLen - 1 && b_side) ? uint32_t('B') : uint32_t(uint8_t(kText[i]));
    m[i / 4] |= ch << (8 * (i % 4));
  }
  uint32_t iv[8];
  b3_iv(iv);
  b3_compress8_at(iv, m, 0, kLen, kB3ChunkStart | kB3ChunkEnd | kB3Root, out);
}

// bind_root (seed.rs:41-58): BLAKE3 keyed by the salt of root || le32(dim)
// || 28 zero bytes.
__device__ void bind_root(const uint32_t* root, uint32_t dim, bool b_side, uint32_t* out) {
  uint32_t salt[8], m[16];
  seed_salt(b_side, salt);
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = root[i];
  m[8] = dim;
  b3_compress8_at(salt, m, 0, 64, kB3Keyed | kB3ChunkStart | kB3ChunkEnd | kB3Root, out);
}

__global__ void commitment_kernel(const CommitArgs a) {
  uint32_t ra[8], rb[8];
  if (a.salted) {
    bind_root(a.root_a, a.dim_a, false, ra);
    bind_root(a.root_b, a.dim_b, true, rb);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ra[i] = a.root_a[i];
      rb[i] = a.root_b[i];
    }
  }
  if (a.routing_root) {  // MoE: A's root absorbs the routing commitment
    uint32_t rr[8], oh[8], hr[8], act[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      rr[i] = a.routing_root[i];
      oh[i] = a.offsets_hash[i];
    }
    hash64(rr, oh, hr);
    hash64(ra, hr, act);
#pragma unroll
    for (int i = 0; i < 8; ++i) ra[i] = act[i];
  }
  uint32_t key[8], cb[8], ca[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) key[i] = a.key[i];
  hash64(key, rb, cb);  // B's seed: BLAKE3(key || B root)
  hash64(cb, ra, ca);   // A's seed: BLAKE3(B's seed || A root)
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a.out_a[i] = ca[i];
    a.out_b[i] = cb[i];
  }
}

bool al4(const void* p) { return reinterpret_cast<uintptr_t>(p) % 4 == 0; }

template <int TPB>
void launch_groups(const TensorHashArgs& a, cudaStream_t s) {
  chunk_group_kernel<TPB><<<a.num_groups, TPB, 0, s>>>(a);
}

}  // namespace
}  // namespace pb2

extern "C" int64_t pb2_required_scratchpad_bytes(int64_t matrix_bytes, int threads_per_block) {
  if (matrix_bytes < 0 || threads_per_block <= 0) return 0;
  const int64_t per_group = int64_t(threads_per_block) * pb2::kChunkBytes;
  return (matrix_bytes + per_group - 1) / per_group * 32;
}

extern "C" int pb2_tensor_hash(const pb2_tensor_hash_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_tensor_hash");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_tensor_hash_params& p = *pp;
  const int tpb = p.threads_per_block;
  if (tpb != 128 && tpb != 256 && tpb != 512) return PB2_ERR_UNSUPPORTED_CONFIG;
  if (p.len <= 0 || !p.data || !p.key || !p.out || !p.roots) return PB2_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(p.data) % 16 != 0 || !al4(p.key) || !al4(p.out) || !al4(p.roots))
    return PB2_ERR_INVALID_ARGUMENT;
  const int64_t groups = pb2_required_scratchpad_bytes(p.len, tpb) / 32;
  if (p.roots_bytes < groups * 32 || groups > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  TensorHashArgs a;
  a.data = p.data;
  a.len = uint64_t(p.len);
  a.chunks = (a.len + kChunkBytes - 1) / kChunkBytes;
  a.num_groups = uint32_t(groups);
  a.key = reinterpret_cast<const uint32_t*>(p.key);
  a.roots = reinterpret_cast<uint32_t*>(p.roots);
  a.out = reinterpret_cast<uint32_t*>(p.out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (tpb == 128) launch_groups<128>(a, s);
  else if (tpb == 256) launch_groups<256>(a, s);
  else launch_groups<512>(a, s);
  if ((st = launch_status())) return st;
  if (a.num_groups > 1) {
    root_fold_kernel<<<1, 1024, 0, s>>>(a);
    if ((st = launch_status())) return st;
  }
  return PB2_OK;
}

// Layer sizes of the tree over `len` bytes; returns the layer count (0 when
// len <= 0 or more than kMerkleMaxLayers) and the total node count.
static int merkle_layout(int64_t len, uint64_t* off, int64_t* total) {
  *total = 0;
  if (len <= 0) return 0;
  uint64_t n = (uint64_t(len) + pb2::kChunkBytes - 1) / pb2::kChunkBytes;
  int layers = 0;
  uint64_t at = 0;
  for (;;) {
    if (layers == pb2::kMerkleMaxLayers) return 0;
    if (off) off[layers] = at;
    ++layers;
    at += n;
    if (n <= 1) break;
    n = n == 2 ? 1 : (n + 1) / 2;
  }
  *total = int64_t(at);
  return layers;
}

extern "C" int64_t pb2_merkle_nodes(int64_t len) {
  int64_t total;
  merkle_layout(len, nullptr, &total);
  return total;
}

extern "C" int pb2_merkle_layers(const pb2_merkle_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_merkle_layers");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_merkle_params& p = *pp;
  if (p.len <= 0 || !p.data || !p.key || !p.nodes) return PB2_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(p.data) % 16 != 0 || !al4(p.key) || !al4(p.nodes))
    return PB2_ERR_INVALID_ARGUMENT;
  MerkleArgs a;
  int64_t total;
  a.layers = merkle_layout(p.len, a.off, &total);
  if (a.layers == 0 || p.nodes_bytes < total * 32) return PB2_ERR_INVALID_ARGUMENT;
  const uint64_t chunks = (uint64_t(p.len) + kChunkBytes - 1) / kChunkBytes;
  const uint64_t groups = (chunks + kMerkleGroup - 1) / kMerkleGroup;
  if (groups > INT32_MAX) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  a.h.data = p.data;
  a.h.len = uint64_t(p.len);
  a.h.chunks = chunks;
  a.h.num_groups = uint32_t(groups);
  a.h.key = reinterpret_cast<const uint32_t*>(p.key);
  a.h.roots = nullptr;
  a.h.out = nullptr;
  a.nodes = reinterpret_cast<uint32_t*>(p.nodes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  merkle_group_kernel<<<unsigned(groups), kMerkleGroup, 0, s>>>(a);
  if ((st = launch_status())) return st;
  if (groups > 1) {
    merkle_top_kernel<<<1, 1024, 0, s>>>(a);
    if ((st = launch_status())) return st;
  }
  return PB2_OK;
}

extern "C" int pb2_commitment_hash_from_merkle_roots(const pb2_commitment_params* pp, void* stream) {
  pb2::NvtxRange nvtx_range("pb2_commitment_hash_from_merkle_roots");
  using namespace pb2;
  if (!pp) return PB2_ERR_INVALID_ARGUMENT;
  const pb2_commitment_params& p = *pp;
  if (!p.A_merkle_root || !p.B_merkle_root || !p.key || !p.A_commitment_hash || !p.B_commitment_hash)
    return PB2_ERR_INVALID_ARGUMENT;
  if ((p.routing_root == nullptr) != (p.offsets_hash == nullptr)) return PB2_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {p.A_merkle_root, p.B_merkle_root, p.key, p.A_commitment_hash,
                        p.B_commitment_hash, p.routing_root, p.offsets_hash};
  for (const void* q : ptrs)
    if (!al4(q)) return PB2_ERR_INVALID_ARGUMENT;
  int st = set_device(p.device);
  if (st) return st;
  CommitArgs a;
  a.root_a = reinterpret_cast<const uint32_t*>(p.A_merkle_root);
  a.root_b = reinterpret_cast<const uint32_t*>(p.B_merkle_root);
  a.key = reinterpret_cast<const uint32_t*>(p.key);
  a.out_a = reinterpret_cast<uint32_t*>(p.A_commitment_hash);
  a.out_b = reinterpret_cast<uint32_t*>(p.B_commitment_hash);
  a.routing_root = reinterpret_cast<const uint32_t*>(p.routing_root);
  a.offsets_hash = reinterpret_cast<const uint32_t*>(p.offsets_hash);
  a.salted = p.salted;
  a.dim_a = p.salted_dim_a;
  a.dim_b = p.salted_dim_b;
  commitment_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}
