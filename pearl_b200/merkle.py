"""Merkle proofs of a hit's rows, built from the tensor already in HBM.

After a hit the miner opens the rows of A and the columns of B that the hit
tile touched: a multi-leaf BLAKE3 Merkle proof over each matrix, zero-padded
to whole 1 KiB chunks (miner_base/block_submission.py:14-62 through
matrix_merkle_tree.py:8-54 onto pearl-blake3/src/merkle.rs:33-175; the Rust
miner's twin is zk-pow/src/ffi/mine.rs:380-430).  The reference copies the
matrix to the host and hashes it there; here ``pb2_merkle_layers`` builds
every layer of the tree on the GPU and only the layers (32 bytes per node)
and the opened chunks come back.  The root equals ``tensor_hash`` of the
same bytes.

Names, argument meaning and errors follow the reference classes:
``MerkleTree`` (over a 1-D byte tensor), ``MatrixMerkleTree`` (over a 2-D
int8 matrix), ``MerkleProof``.  Proof verification is the consensus node's
job and is not part of the miner's path.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from .pearl_gemm_interface import _device_index, _fail, _stream

MERKLE_LEAF_SIZE = 1024  # BLAKE3 chunk (merkle.rs:9 CHUNK_LEN)
DIGEST_SIZE = 32


def padded_chunk_len(raw_len: int) -> int:
    """``raw_len`` rounded up to whole chunks (merkle.rs:15-17)."""
    return -(-int(raw_len) // MERKLE_LEAF_SIZE) * MERKLE_LEAF_SIZE


def merkle_layer_sizes(length: int) -> list[int]:
    """Node count of each layer, leaves first (merkle.rs:62-75): one node per
    chunk; while a layer has more than two nodes the next has ceil(n / 2); a
    two-node layer is followed by the root; one chunk is its own root."""
    n = padded_chunk_len(length) // MERKLE_LEAF_SIZE
    if n == 0:
        return []
    sizes = [n]
    while n > 1:
        n = (n + 1) // 2
        sizes.append(n)
    return sizes


@dataclass
class MerkleProof:
    """pearl-blake3/src/merkle.rs:183-191: the opened chunks (sorted, unique
    leaf indices), the leaf count, the root and the sibling CVs in the order
    the level walk meets them."""
    leaf_data: list[bytes]
    leaf_indices: list[int]
    total_leaves: int
    root: bytes
    siblings: list[bytes] = field(default_factory=list)


def multileaf_proof(layers: list[np.ndarray], leaf_indices, leaf_chunk) -> MerkleProof:
    """MerkleTree::get_multileaf_proof (merkle.rs:104-155) over host copies of
    the layers ((n, 32) uint8 arrays, leaves first); ``leaf_chunk(i)`` returns
    chunk i's 1 KiB."""
    if len(leaf_indices) == 0:
        raise ValueError("leaf_indices must be non-empty")
    unique = sorted(set(int(i) for i in leaf_indices))
    total = len(layers[0])
    if unique[0] < 0 or unique[-1] >= total:
        raise ValueError("leaf index out of bounds")
    siblings: list[bytes] = []
    cur, level_len, level = unique, total, 0
    while level_len > 1 and cur:
        nodes, present = layers[level], set(cur)
        for i in cur:
            if i % 2 == 1:
                if i - 1 not in present:
                    siblings.append(nodes[i - 1].tobytes())
            elif i + 1 not in present and i + 1 < level_len:
                siblings.append(nodes[i + 1].tobytes())
        cur = sorted(set(i // 2 for i in cur))
        level_len = (level_len + 1) // 2
        level += 1
    return MerkleProof([leaf_chunk(i) for i in unique], unique, total, layers[-1][0].tobytes(), siblings)


def _key_tensor(key: bytes, device: torch.device) -> torch.Tensor:
    return torch.frombuffer(bytearray(key), dtype=torch.uint8).to(device)


def merkle_layers(data: torch.Tensor, key, nodes: torch.Tensor) -> None:
    """Every layer of the keyed tree over ``data``'s bytes into ``nodes``
    (uint8, at least ``pb2_merkle_nodes(len) * 32`` bytes) on the current
    stream.  ``data`` is a contiguous CUDA tensor, ``key`` a 32-byte uint8
    CUDA tensor."""
    for t, name in ((data, "data"), (key, "key"), (nodes, "nodes")):
        if not t.is_cuda:
            _fail(f"{name} must be on CUDA")
        if not t.is_contiguous():
            _fail(f"{name} must be contiguous")
    if key.dtype != torch.uint8 or key.numel() != DIGEST_SIZE:
        _fail("key must be 32 uint8 bytes")
    if nodes.dtype != torch.uint8:
        _fail("nodes must be uint8")
    length = data.numel() * data.element_size()
    if length == 0:
        _fail("data must be non-empty")
    if data.data_ptr() % 16 != 0:
        _fail("data must be 16-byte aligned")
    p = _lib.MerkleParams(device=_device_index(data), data=data.data_ptr(), len=length,
                          key=key.data_ptr(), nodes=nodes.data_ptr(), nodes_bytes=nodes.numel())
    with torch.cuda.device(data.device):
        _lib.call("pb2_merkle_layers", p, _stream(data.device), "merkle_layers")


class MerkleTree:
    """Keyed BLAKE3 Merkle tree of a CUDA tensor's bytes zero-padded to whole
    chunks (merkle.rs:33-81 on pad_to_chunk_boundary, :22-27).  The layers
    are built on the tensor's GPU; the tree keeps a reference to the tensor
    for the opened chunks."""

    def __init__(self, data: torch.Tensor, key: bytes):
        if len(key) != DIGEST_SIZE:
            raise ValueError(f"Expected 32-byte key, got {len(key)} bytes")
        if not data.is_cuda:
            _fail("data must be on CUDA")
        self._key = bytes(key)
        self._data = data.contiguous().view(-1).view(torch.uint8)
        self._len = self._data.numel()
        sizes = merkle_layer_sizes(self._len)
        total = int(_lib.load().pb2_merkle_nodes(self._len))
        if total != sum(sizes):
            _fail("merkle layout mismatch between host and library")
        self._sizes = sizes
        self._nodes = torch.empty(max(total, 1) * DIGEST_SIZE, dtype=torch.uint8, device=data.device)
        if self._len:
            merkle_layers(self._data, _key_tensor(self._key, data.device), self._nodes)
        self._host_layers: list[np.ndarray] | None = None

    def key(self) -> bytes:
        return self._key

    def _layers(self) -> list[np.ndarray]:
        if self._host_layers is None:
            flat = self._nodes.cpu().numpy().reshape(-1, DIGEST_SIZE)
            out, off = [], 0
            for s in self._sizes:
                out.append(flat[off:off + s])
                off += s
            self._host_layers = out
        return self._host_layers

    @property
    def root(self) -> bytes:
        if not self._sizes:
            return bytes(DIGEST_SIZE)
        return self._layers()[-1][0].tobytes()

    @property
    def leaf_hashes(self) -> list[bytes]:
        if not self._sizes:
            return []
        return [r.tobytes() for r in self._layers()[0]]

    def num_leaves(self) -> int:
        return self._sizes[0] if self._sizes else 0

    def _chunk(self, i: int) -> bytes:
        lo = i * MERKLE_LEAF_SIZE
        hi = min(lo + MERKLE_LEAF_SIZE, self._len)
        return self._data[lo:hi].cpu().numpy().tobytes().ljust(MERKLE_LEAF_SIZE, b"\0")

    def get_multileaf_proof(self, leaf_indices) -> MerkleProof:
        """MerkleTree::get_multileaf_proof (merkle.rs:104-155)."""
        if not self._sizes:
            raise ValueError("empty tree")
        return multileaf_proof(self._layers(), leaf_indices, self._chunk)

    @staticmethod
    def compute_leaf_indices_from_rows(row_indices, shape) -> list[int]:
        """Chunks holding the given rows of a row-major byte matrix
        (merkle.rs:158-174)."""
        cols = int(shape[1])
        out = set()
        for row in row_indices:
            first = (int(row) * cols) // MERKLE_LEAF_SIZE
            last = ((int(row) + 1) * cols - 1) // MERKLE_LEAF_SIZE
            out.update(range(first, last + 1))
        return sorted(out)


class MatrixMerkleTree:
    """miner_base/matrix_merkle_tree.py:8-54 on the GPU: the tree of a 2-D
    int8 matrix (A, or Bᵀ in its (N, K) storage) with the same checks."""

    LEAF_SIZE = MERKLE_LEAF_SIZE

    def __init__(self, tensor: torch.Tensor, key: bytes):
        if tensor.numel() == 0:
            raise ValueError("tensor must be non-empty")
        if tensor.dim() != 2:
            raise ValueError(f"Expected 2D tensor, got {tensor.dim()}D tensor")
        if tensor.dtype != torch.int8:
            raise ValueError(f"Expected int8 tensor, got {tensor.dtype}")
        if len(key) != 32:
            raise ValueError(f"Expected 32-byte key, got {len(key)} bytes")
        self.tensor_shape = tuple(tensor.shape)
        self._tree = MerkleTree(tensor, key)

    @property
    def root(self) -> bytes:
        return self._tree.root

    @property
    def leaf_hashes(self) -> list[bytes]:
        return self._tree.leaf_hashes

    def leaf_indices_from_rows(self, row_indices) -> list[int]:
        return MerkleTree.compute_leaf_indices_from_rows(row_indices, self.tensor_shape)

    def get_multileaf_proof(self, leaf_indices) -> MerkleProof:
        return self._tree.get_multileaf_proof(leaf_indices)


def open_rows(tensor: torch.Tensor, key: bytes, row_indices) -> MerkleProof:
    """The per-matrix step of create_proof (block_submission.py:25-40): the
    proof of the chunks holding ``row_indices`` of ``tensor``."""
    tree = MatrixMerkleTree(tensor, key)
    return tree.get_multileaf_proof(tree.leaf_indices_from_rows(row_indices))


@dataclass
class MoERoutingProof:
    """The routing part of a MoE proof (block_submission.py:64-88,
    MoEProofParams): which expert's segment of the routed token list the hit
    used, and the Merkle proof of the opened routing entries."""
    e: int
    top_k: int
    expert_idx: int
    routing_end_offsets: list[int]
    inner_a_rows: list[int]
    routing_proof: MerkleProof


def moe_routing_proof(routing_data: torch.Tensor, routing_end_offsets, expert_idx: int, inner_a_rows,
                      key: bytes, num_experts: int, top_k: int) -> MoERoutingProof:
    """_build_moe_proof_params (block_submission.py:64-88) on the GPU copy of
    the routing data: each u32 entry of ``routing_data`` (the expert-sorted
    token list of build_routing_data) is one 4-byte row of the committed
    matrix; the expert's segment starts at the previous expert's exclusive
    end; the opened rows are that start plus the hit's rows inside the
    expert's A slice."""
    if routing_data.dtype not in (torch.int32, torch.uint32):
        raise ValueError("routing_data must be a 32-bit tensor")
    offsets = [int(x) for x in routing_end_offsets]
    if not 0 <= expert_idx < len(offsets):
        raise ValueError("expert_idx out of range")
    rows = routing_data.contiguous().view(torch.int8).reshape(-1, 4)
    tree = MatrixMerkleTree(rows, key)
    start = 0 if expert_idx == 0 else offsets[expert_idx - 1]
    global_rows = [start + int(r) for r in inner_a_rows]
    proof = tree.get_multileaf_proof(tree.leaf_indices_from_rows(global_rows))
    return MoERoutingProof(num_experts, top_k, expert_idx, offsets, [int(r) for r in inner_a_rows], proof)
