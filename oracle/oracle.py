"""ctypes/numpy front end of ``pearl_oracle.c`` (a CPU restatement of the
reference's Rust protocol code in ``zk-pow``).

TEST INFRASTRUCTURE ONLY -- the parity checker and the timed CPU baseline.
Every function names the reference code it restates.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libpearl_oracle.so")
_lib = None

ROWS_PATTERN = [0, 8]
COLS_PATTERN = [c + d for c in range(0, 256, 8) for d in (0, 1)]


def build() -> str:
    """Compile the oracle shared library with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        i8p = ctypes.POINTER(ctypes.c_int8)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        i32p = ctypes.POINTER(ctypes.c_int32)
        i64p = ctypes.POINTER(ctypes.c_int64)
        i64 = ctypes.c_int64
        L.po_blake3.argtypes = [u8p, ctypes.c_size_t, u8p, u8p]
        L.po_blake3_compress.argtypes = [u32p, u32p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, u32p]
        L.po_noise_dense.argtypes = [u8p, ctypes.c_int, i64, i64, i8p]
        L.po_noise_pairs.argtypes = [u8p, ctypes.c_int, i64, i64, u8p]
        L.po_noise_operand.argtypes = [i8p, i8p, i64, i64, i64, u8p, i8p]
        L.po_times_pairs.argtypes = [i8p, i64, i64, i64, u8p, i32p]
        L.po_jackpot_tile.argtypes = [i8p, i8p, i64, i64, i64p, ctypes.c_int, i64p, ctypes.c_int, u32p]
        L.po_jackpot_hash.argtypes = [u32p, u8p, u32p]
        L.po_u256_le.argtypes = [u32p, u32p]
        L.po_mine_tiles.argtypes = [i8p, i8p, i64, i64, i64, i64, u8p, u32p, i64, i64, u32p, u32p, u8p]
        L.po_mine_tiles_f32.argtypes = L.po_mine_tiles.argtypes
        L.po_hash_activations.argtypes = [u8p, u8p, u32p, i64, u8p, u8p]
        L.po_commitment.argtypes = [u8p, u8p, u8p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32,
                                    u8p, u32p, i64, u8p, u8p]
        L.po_tensor_hash.argtypes = [u8p, i64, u8p, u8p]
        L.po_merkle_nodes.argtypes = [i64]
        L.po_merkle_nodes.restype = i64
        L.po_merkle_layers.argtypes = [u8p, i64, u8p, u8p]
        L.po_chunk_cv.argtypes = [u8p, u8p, ctypes.c_uint64, u8p]
        L.po_parent_cv.argtypes = [u8p, u8p, u8p, ctypes.c_int, u8p]
        L.po_num_threads.restype = ctypes.c_int
        L.po_set_num_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray, ct):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ct))


def _bytes32(x) -> np.ndarray:
    a = np.frombuffer(bytes(x), dtype=np.uint8).copy() if not isinstance(x, np.ndarray) else x
    a = np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)
    assert a.size == 32
    return a


# ---------------------------------------------------------------- BLAKE3 ---
def blake3(data: bytes, key: bytes | None = None) -> bytes:
    """blake3 / keyed blake3 digest (pearl-blake3/src/hasher.rs:183-188)."""
    d = np.frombuffer(bytes(data), dtype=np.uint8).copy() if len(data) else np.zeros(1, np.uint8)
    out = np.zeros(32, np.uint8)
    k = _p(_bytes32(key), ctypes.c_uint8) if key is not None else None
    lib().po_blake3(_p(d, ctypes.c_uint8), len(data), k, _p(out, ctypes.c_uint8))
    return out.tobytes()


def blake3_compress(cv, block, counter, block_len, flags) -> np.ndarray:
    cv = np.ascontiguousarray(cv, np.uint32)
    block = np.ascontiguousarray(block, np.uint32)
    out = np.zeros(16, np.uint32)
    lib().po_blake3_compress(_p(cv, ctypes.c_uint32), _p(block, ctypes.c_uint32), counter, block_len,
                             flags, _p(out, ctypes.c_uint32))
    return out


# ----------------------------------------------------------------- noise ---
def noise_dense(key: bytes, which: str, rows: int, r: int) -> np.ndarray:
    """EAL (which='A') or EBR (which='B'), rows x r int8 in [-32, 32)
    (zk-pow/src/circuit/pearl_noise.rs:61-80)."""
    out = np.zeros((rows, r), np.int8)
    lib().po_noise_dense(_p(_bytes32(key), ctypes.c_uint8), int(which == "B"), rows, r,
                         _p(out, ctypes.c_int8))
    return out


def noise_pairs(key: bytes, which: str, k: int, r: int) -> np.ndarray:
    """(k, 2) uint8 index pairs: +1 at [:,0], -1 at [:,1]
    (pearl_noise.rs:90-116)."""
    out = np.zeros((k, 2), np.uint8)
    lib().po_noise_pairs(_p(_bytes32(key), ctypes.c_uint8), int(which == "B"), k, r,
                         _p(out, ctypes.c_uint8))
    return out


def pairs_to_r_major(pairs: np.ndarray, r: int) -> np.ndarray:
    """(k, r) int8 matrix with +1/-1 per row: the reference's *_R_major form."""
    k = pairs.shape[0]
    m = np.zeros((k, r), np.int8)
    m[np.arange(k), pairs[:, 0]] = 1
    m[np.arange(k), pairs[:, 1]] = -1
    return m


def noise_operand(x: np.ndarray, el: np.ndarray, pairs: np.ndarray) -> np.ndarray:
    """x + el . S^T with S the pair matrix (ApEA / BpEB), int8 wrap."""
    x = np.ascontiguousarray(x, np.int8)
    el = np.ascontiguousarray(el, np.int8)
    pairs = np.ascontiguousarray(pairs, np.uint8)
    rows, k = x.shape
    r = el.shape[1]
    out = np.zeros_like(x)
    lib().po_noise_operand(_p(x, ctypes.c_int8), _p(el, ctypes.c_int8), rows, k, r,
                           _p(pairs, ctypes.c_uint8), _p(out, ctypes.c_int8))
    return out


def times_pairs(x: np.ndarray, pairs: np.ndarray, r: int) -> np.ndarray:
    """x . S (rows x r, int32): AxEBL (x=A, S=EBL) and EARxBpEB (x=BpEB, S=EAR)."""
    x = np.ascontiguousarray(x, np.int8)
    pairs = np.ascontiguousarray(pairs, np.uint8)
    rows, k = x.shape
    out = np.zeros((rows, r), np.int32)
    lib().po_times_pairs(_p(x, ctypes.c_int8), rows, k, r, _p(pairs, ctypes.c_uint8),
                         _p(out, ctypes.c_int32))
    return out


# --------------------------------------------------------------- jackpot ---
def hash_tile_origin(m: int, n: int, t: int) -> tuple[int, int]:
    """(row offset, col offset) of protocol hash tile t (row-major tile order)."""
    tcols = n // 64
    trow, tcol = divmod(t, tcols)
    return 16 * (trow // 8) + trow % 8, 256 * (tcol // 4) + 2 * (tcol % 4)


def num_hash_tiles(m: int, n: int) -> int:
    return (m // 2) * (n // 64)


def jackpot_tile(ap, bp, k, r, rows, cols) -> np.ndarray:
    rows = np.ascontiguousarray(rows, np.int64)
    cols = np.ascontiguousarray(cols, np.int64)
    out = np.zeros(16, np.uint32)
    lib().po_jackpot_tile(_p(ap, ctypes.c_int8), _p(bp, ctypes.c_int8), k, r, _p(rows, ctypes.c_int64),
                          len(rows), _p(cols, ctypes.c_int64), len(cols), _p(out, ctypes.c_uint32))
    return out


def jackpot_hash(transcript, key: bytes) -> np.ndarray:
    t = np.ascontiguousarray(transcript, np.uint32)
    out = np.zeros(8, np.uint32)
    lib().po_jackpot_hash(_p(t, ctypes.c_uint32), _p(_bytes32(key), ctypes.c_uint8),
                          _p(out, ctypes.c_uint32))
    return out


def target_words(target: int) -> np.ndarray:
    return np.array([(target >> (32 * i)) & 0xFFFFFFFF for i in range(8)], np.uint32)


@dataclass
class MineResult:
    transcripts: np.ndarray  # (tiles, 16) uint32
    digests: np.ndarray  # (tiles, 8) uint32
    hits: np.ndarray  # (tiles,) bool
    tile_begin: int


def mine_tiles(ap: np.ndarray, bp: np.ndarray, r: int, key: bytes, target: int,
               tile_begin: int = 0, tile_end: int | None = None, acc_f32: bool = False) -> MineResult:
    """Transcripts, digests and hit flags of protocol hash tiles
    [tile_begin, tile_end) for noised operands ap (m x k) and bp (n x k)
    (zk-pow/src/ffi/mine.rs:86-110).  acc_f32 folds the float32 bit patterns
    of the accumulators instead of their int32 words (the FP8 mined GEMM of
    this build; exact for integer-valued operands while |sums| < 2^24)."""
    ap = np.ascontiguousarray(ap, np.int8)
    bp = np.ascontiguousarray(bp, np.int8)
    m, k = ap.shape
    n = bp.shape[0]
    assert m % 16 == 0 and n % 256 == 0, "threads_partition needs m%16==0, n%256==0"
    if tile_end is None:
        tile_end = num_hash_tiles(m, n)
    cnt = tile_end - tile_begin
    tr = np.zeros((cnt, 16), np.uint32)
    dg = np.zeros((cnt, 8), np.uint32)
    hits = np.zeros(cnt, np.uint8)
    tw = target_words(target)
    fn = lib().po_mine_tiles_f32 if acc_f32 else lib().po_mine_tiles
    fn(_p(ap, ctypes.c_int8), _p(bp, ctypes.c_int8), m, n, k, r, _p(_bytes32(key), ctypes.c_uint8),
       _p(tw, ctypes.c_uint32), tile_begin, tile_end, _p(tr, ctypes.c_uint32), _p(dg, ctypes.c_uint32),
       _p(hits, ctypes.c_uint8))
    return MineResult(tr, dg, hits.astype(bool), tile_begin)


def hit_set(res: MineResult, m: int, n: int) -> set[tuple[int, int]]:
    return {hash_tile_origin(m, n, res.tile_begin + int(i)) for i in np.nonzero(res.hits)[0]}


# ------------------------------------------------------------ commitment ---
def commitment(job_key: bytes, hash_a: bytes, hash_b: bytes, salted_dims=None,
               routing_root: bytes | None = None, offsets=None) -> tuple[bytes, bytes]:
    """(b_noise_seed, a_noise_seed) -- zk-pow/src/api/proof_utils.rs:361-372,
    api/seed.rs:20-58, proof_utils.rs:34-45."""
    bs = np.zeros(32, np.uint8)
    as_ = np.zeros(32, np.uint8)
    salted = salted_dims is not None
    m, n = salted_dims if salted else (0, 0)
    off = np.ascontiguousarray(offsets if offsets is not None else np.zeros(0), np.uint32)
    rr = _p(_bytes32(routing_root), ctypes.c_uint8) if routing_root is not None else None
    lib().po_commitment(_p(_bytes32(job_key), ctypes.c_uint8), _p(_bytes32(hash_a), ctypes.c_uint8),
                        _p(_bytes32(hash_b), ctypes.c_uint8), int(salted), m, n, rr,
                        _p(off, ctypes.c_uint32) if off.size else None, off.size,
                        _p(bs, ctypes.c_uint8), _p(as_, ctypes.c_uint8))
    return bs.tobytes(), as_.tobytes()


def tensor_hash(data: np.ndarray, key: bytes) -> bytes:
    """Keyed BLAKE3 of the bytes zero-padded to 1 KiB chunks
    (pearl-blake3/src/merkle.rs:15-27; zk-pow/src/ffi/mine.rs:448-452)."""
    d = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    out = np.zeros(32, np.uint8)
    lib().po_tensor_hash(_p(d, ctypes.c_uint8) if d.size else None, d.size,
                         _p(_bytes32(key), ctypes.c_uint8), _p(out, ctypes.c_uint8))
    return out.tobytes()


# ----------------------------------------------------------------- merkle ---
def merkle_layers(data: np.ndarray, key: bytes) -> list[np.ndarray]:
    """Layers (leaves first) of the BLAKE3 Merkle tree over the bytes
    zero-padded to 1 KiB chunks (pearl-blake3/src/merkle.rs:43-81 on
    pad_to_chunk_boundary, :15-27); each layer is an (n, 32) uint8 array."""
    d = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    total = int(lib().po_merkle_nodes(d.size))
    nodes = np.zeros((max(total, 1), 32), np.uint8)
    if d.size:
        lib().po_merkle_layers(_p(d, ctypes.c_uint8), d.size, _p(_bytes32(key), ctypes.c_uint8),
                               _p(nodes, ctypes.c_uint8))
    sizes, n = [], (d.size + 1023) // 1024
    if n:
        sizes.append(n)
        while n > 2:
            n = (n + 1) // 2
            sizes.append(n)
        if n == 2:
            sizes.append(1)
    out, off = [], 0
    for s in sizes:
        out.append(nodes[off:off + s])
        off += s
    return out


def multileaf_proof(layers: list[np.ndarray], padded: bytes, leaf_indices) -> dict:
    """MerkleTree::get_multileaf_proof (pearl-blake3/src/merkle.rs:104-155):
    sorted unique leaves, their 1 KiB chunks, and the sibling CVs in the
    order the level walk meets them."""
    unique = sorted(set(int(i) for i in leaf_indices))
    total = len(layers[0])
    assert unique and unique[-1] < total
    leaf_data = [bytes(padded[i * 1024:(i + 1) * 1024]).ljust(1024, b"\0") for i in unique]
    siblings, cur, level_len, level = [], unique, total, 0
    while level_len > 1 and cur:
        nodes, cs = layers[level], set(cur)
        for i in cur:
            if i % 2 == 1:
                if i - 1 not in cs:
                    siblings.append(nodes[i - 1].tobytes())
            elif i + 1 not in cs and i + 1 < level_len:
                siblings.append(nodes[i + 1].tobytes())
        cur = sorted(set(i // 2 for i in cur))
        level_len = (level_len + 1) // 2
        level += 1
    return {"leaf_data": leaf_data, "leaf_indices": unique, "total_leaves": total,
            "root": layers[-1][0].tobytes(), "siblings": siblings}


def chunk_cv(key: bytes, chunk: bytes, index: int) -> bytes:
    c = np.frombuffer(bytes(chunk), np.uint8).copy()
    assert c.size == 1024
    out = np.zeros(32, np.uint8)
    lib().po_chunk_cv(_p(_bytes32(key), ctypes.c_uint8), _p(c, ctypes.c_uint8), index,
                      _p(out, ctypes.c_uint8))
    return out.tobytes()


def parent_cv(key: bytes, left: bytes, right: bytes, root: bool) -> bytes:
    l_, r_ = _bytes32(left), _bytes32(right)
    out = np.zeros(32, np.uint8)
    lib().po_parent_cv(_p(_bytes32(key), ctypes.c_uint8), _p(l_, ctypes.c_uint8),
                       _p(r_, ctypes.c_uint8), int(root), _p(out, ctypes.c_uint8))
    return out.tobytes()


def proof_root(proof: dict, key: bytes):
    """MerkleProof::compute_root (pearl-blake3/src/merkle.rs:222-289): the
    root rebuilt from the leaf chunks and the siblings, None when the proof
    has the wrong shape."""
    idx = proof["leaf_indices"]
    if not idx:
        return None
    cur = {i: chunk_cv(key, d, i) for i, d in zip(idx, proof["leaf_data"])}
    level_len = proof["total_leaves"]
    if level_len == 1:
        if proof["siblings"]:
            return None
        # the single leaf is the root: the keyed hash of its chunk
        return blake3(proof["leaf_data"][0], key)
    sib = iter(proof["siblings"])
    try:
        while level_len > 2:
            nxt = {}
            for i in sorted(cur):
                cv = cur[i]
                if i % 2 == 0:
                    if i + 1 in cur:
                        nxt[i // 2] = parent_cv(key, cv, cur[i + 1], False)
                    elif i + 1 < level_len:
                        nxt[i // 2] = parent_cv(key, cv, next(sib), False)
                    else:
                        nxt[i // 2] = cv
                elif i - 1 not in cur:
                    nxt[i // 2] = parent_cv(key, next(sib), cv, False)
            cur, level_len = nxt, (level_len + 1) // 2
        left = cur[0] if 0 in cur else next(sib)
        right = cur[1] if 1 in cur else next(sib)
    except StopIteration:
        return None
    if next(sib, None) is not None:
        return None
    return parent_cv(key, left, right, True)


# ---------------------------------------------------------------- routing ---
def routing_order(topk_ids: np.ndarray, num_experts: int):
    """(routing_data, slot_indices, routing_offsets) of build_routing_data
    (miner/pearl-gemm/csrc/moe/build_routing_data.cu:40-77): flat slots
    stably sorted by 8-bit expert id, their tokens, and per-expert exclusive
    ends."""
    ids = np.ascontiguousarray(topk_ids, np.int64)
    top_k = ids.shape[1]
    keys = ids.reshape(-1) & 0xFF
    slots = np.argsort(keys, kind="stable").astype(np.int32)
    offsets = np.array([(keys <= e).sum() for e in range(num_experts)], np.int32)
    return (slots // top_k).astype(np.int32), slots, offsets


def num_threads() -> int:
    return lib().po_num_threads()


def set_num_threads(n: int) -> None:
    lib().po_set_num_threads(n)


# ----------------------------------------------------- whole noisy GEMM ----
@dataclass
class NoisyProblem:
    A: np.ndarray
    B: np.ndarray
    EAL: np.ndarray
    EBR: np.ndarray
    EAR_pairs: np.ndarray
    EBL_pairs: np.ndarray
    ApEA: np.ndarray
    BpEB: np.ndarray
    AxEBL: np.ndarray
    EARxBpEB: np.ndarray


def noisy_problem(A: np.ndarray, B: np.ndarray, key_a: bytes, key_b: bytes, r: int) -> NoisyProblem:
    """Noise factors and noised operands for A (m x k), B (n x k)
    (zk-pow/src/circuit/pearl_noise.rs:118-160, mine.rs:61-85)."""
    m, k = A.shape
    n = B.shape[0]
    EAL = noise_dense(key_a, "A", m, r)
    EBR = noise_dense(key_b, "B", n, r)
    EAR = noise_pairs(key_a, "A", k, r)
    EBL = noise_pairs(key_b, "B", k, r)
    ApEA = noise_operand(A, EAL, EAR)
    BpEB = noise_operand(B, EBR, EBL)
    AxEBL = times_pairs(A, EBL, r)
    EARxBpEB = times_pairs(BpEB, EAR, r)
    return NoisyProblem(A, B, EAL, EBR, EAR, EBL, ApEA, BpEB, AxEBL, EARxBpEB)
