"""Host-side parts of PlainProof assembly (pearl_b200.proof): the commitment
key (CommitmentHasher.get_key, commitment_hash.py:36-37) and the dataclass
fields a caller copies into the pearl_mining proof types."""
import dataclasses

import pytest

from oracle import oracle as O
from pearl_b200 import proof as PF


def test_commitment_key_is_blake3_of_header_and_config():
    header, config = bytes(range(80)), b"cfg" + bytes(20)
    assert PF.commitment_key(header, config) == O.blake3(header + config)
    key = bytes(range(32))
    assert PF.commitment_key(hash_key=key) == key
    with pytest.raises(ValueError):
        PF.commitment_key(hash_key=bytes(16))
    with pytest.raises(ValueError):
        PF.commitment_key(header)


def test_proof_dataclass_fields_match_the_reference_types():
    # pearl_mining.PlainProof / MatrixMerkleProof / MoEProofParams and the
    # gateway's OpenedBlockInfo / MoEBlockInfo field names.
    assert [f.name for f in dataclasses.fields(PF.PlainProof)] == [
        "m", "n", "k", "noise_rank", "a_merkle_proof", "bt_merkle_proof", "moe"]
    assert [f.name for f in dataclasses.fields(PF.MatrixMerkleProof)] == ["proof", "row_indices"]
    assert [f.name for f in dataclasses.fields(PF.MoEProofParams)] == [
        "e", "top_k", "expert_idx", "routing_end_offsets", "inner_a_rows", "routing_proof"]
    assert [f.name for f in dataclasses.fields(PF.OpenedBlock)] == [
        "A_row_indices", "B_column_indices", "A", "B_t", "noise_rank", "moe"]
    assert [f.name for f in dataclasses.fields(PF.MoEBlock)] == [
        "expert_index", "num_experts", "n_per_expert", "top_k", "inner_a_rows", "inner_b_cols", "routing_data",
        "expert_routing_offsets"]
