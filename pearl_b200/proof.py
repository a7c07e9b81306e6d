"""PlainProof assembly: from a GPU hit to the proof object the gateway submits.

Restates ``create_proof`` and ``_build_moe_proof_params`` of the reference
miner (miner/miner-base/src/miner_base/block_submission.py:14-88) over this
package's Merkle trees, which are built on the GPU from the matrices already
in HBM (``pearl_b200.merkle``).  The reference's proof types come from the
``pearl_mining`` extension (``PlainProof``, ``MatrixMerkleProof``,
``MoEProofParams``) and its input from the gateway's dataclasses
(``OpenedBlockInfo``, ``MoEBlockInfo``,
miner/pearl-gateway/src/pearl_gateway/comm/dataclasses.py:133-173); the
dataclasses below carry the same fields under the same names, so a caller
copies them field by field into the extension's types.

The commitment key is ``CommitmentHasher.get_key`` (commitment_hash.py:36-37):
BLAKE3 of the incomplete block header followed by the serialized mining
configuration.  The serialization belongs to the ``pearl_mining`` extension
(``MiningConfiguration.to_bytes``), so the caller passes either those bytes
or the job's key itself (the gateway's job already carries it).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .helpers import HostSignalHeader, extract_indices
from .merkle import MatrixMerkleTree, MerkleProof, MoERoutingProof, moe_routing_proof
from .shard import job_key

# The reference's name for the routing part of a MoE proof.
MoEProofParams = MoERoutingProof


@dataclass
class MoEBlock:
    """The MoE fields of an opened block (MoEBlockInfo): the hit's expert,
    the expert count, the per-expert output width, top-k, the hit's rows of
    the expert's A slice and columns of its B slice, the expert-sorted token
    list (build_routing_data's routing_data) and the per-expert exclusive end
    offsets of that list."""
    expert_index: int
    num_experts: int
    n_per_expert: int
    top_k: int
    inner_a_rows: list[int]
    inner_b_cols: list[int]
    routing_data: torch.Tensor
    expert_routing_offsets: list[int]


@dataclass
class OpenedBlock:
    """What a hit opens (OpenedBlockInfo): the A rows and B columns of the hit
    tile, the non-noised operands (A as (m, k); B_t as (n, k), the weight in
    the layout the GEMM reads it), the noise rank and, for a MoE layer, its
    routing fields."""
    A_row_indices: list[int]
    B_column_indices: list[int]
    A: torch.Tensor
    B_t: torch.Tensor
    noise_rank: int
    moe: MoEBlock | None = None


@dataclass
class MatrixMerkleProof:
    """pearl_mining.MatrixMerkleProof: a multi-leaf proof and the matrix rows
    it opens."""
    proof: MerkleProof
    row_indices: list[int]


@dataclass
class PlainProof:
    """pearl_mining.PlainProof: the GEMM's shape (n per expert for MoE), the
    noise rank, the proofs of A's opened rows and of B_t's opened rows, and
    the MoE routing proof."""
    m: int
    n: int
    k: int
    noise_rank: int
    a_merkle_proof: MatrixMerkleProof
    bt_merkle_proof: MatrixMerkleProof
    moe: MoEProofParams | None = None


def commitment_key(incomplete_header_bytes: bytes | None = None, mining_config_bytes: bytes | None = None,
                   *, hash_key: bytes | None = None) -> bytes:
    """The job's 32-byte commitment key: ``hash_key`` when given, else
    BLAKE3(incomplete header || serialized mining configuration)."""
    if hash_key is not None:
        if len(hash_key) != 32:
            raise ValueError("hash_key must be 32 bytes")
        return bytes(hash_key)
    if incomplete_header_bytes is None or mining_config_bytes is None:
        raise ValueError("pass hash_key, or the incomplete header and the serialized mining configuration")
    return job_key(incomplete_header_bytes, mining_config_bytes)


def build_moe_proof_params(moe: MoEBlock, hash_key: bytes) -> MoEProofParams:
    """_build_moe_proof_params (block_submission.py:64-88): the routing data
    as a matrix of 4-byte rows, the expert's segment starting at the previous
    expert's exclusive end, the hit's rows opened at that start."""
    return moe_routing_proof(moe.routing_data, moe.expert_routing_offsets, moe.expert_index, moe.inner_a_rows,
                             hash_key, moe.num_experts, moe.top_k)


def create_proof(opened: OpenedBlock, incomplete_header_bytes: bytes | None = None,
                 mining_config_bytes: bytes | None = None, *, hash_key: bytes | None = None) -> PlainProof:
    """create_proof (block_submission.py:14-61): Merkle trees of A and of B_t
    under the job's key, multi-leaf proofs of the chunks holding the opened
    rows of each, the shape (for MoE, n is the per-expert width while B_t
    stacks every expert) and the routing proof."""
    A, B_t = opened.A, opened.B_t
    if A is None or B_t is None:
        raise ValueError("A and B must be provided")
    if A.dim() != 2 or B_t.dim() != 2:
        raise ValueError("A and B_t must be matrices")
    m, k = A.shape
    n, k2 = B_t.shape
    if k != k2:
        raise ValueError(f"Common dimension mismatch: {k} != {k2}")
    key = commitment_key(incomplete_header_bytes, mining_config_bytes, hash_key=hash_key)
    a_tree = MatrixMerkleTree(A, key)
    b_tree = MatrixMerkleTree(B_t, key)
    a_rows = [int(r) for r in opened.A_row_indices]
    b_rows = [int(c) for c in opened.B_column_indices]
    a_proof = MatrixMerkleProof(a_tree.get_multileaf_proof(a_tree.leaf_indices_from_rows(a_rows)), a_rows)
    b_proof = MatrixMerkleProof(b_tree.get_multileaf_proof(b_tree.leaf_indices_from_rows(b_rows)), b_rows)
    moe_params = None
    if opened.moe is not None:
        moe_params = build_moe_proof_params(opened.moe, key)
        n = opened.moe.n_per_expert
    return PlainProof(m=int(m), n=int(n), k=int(k), noise_rank=int(opened.noise_rank), a_merkle_proof=a_proof,
                      bt_merkle_proof=b_proof, moe=moe_params)


def opened_block_from_hit(header: HostSignalHeader, A: torch.Tensor, B_t: torch.Tensor, noise_rank: int,
                          moe: MoEBlock | None = None) -> OpenedBlock:
    """The opened block of the hit a pinned header reports: its A rows and B
    columns as extract_indices gives them (helpers.py:73-82), over the
    non-noised operands the GEMM read."""
    idx = extract_indices(header)
    return OpenedBlock(A_row_indices=list(idx.A_row_indices), B_column_indices=list(idx.B_column_indices), A=A,
                       B_t=B_t, noise_rank=int(noise_rank), moe=moe)
