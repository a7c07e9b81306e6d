"""Merkle proofs of a hit's rows: the oracle restatement of
pearl-blake3/src/merkle.rs pinned against the `blake3` package (the
reference's own BLAKE3 dependency) and the structural facts of merkle.rs's
tests, and the host side of pearl_b200.merkle (layer layout, proof walk, row
to leaf mapping, argument checks) run on oracle-built layers.  No GPU."""
import random

import numpy as np
import pytest
import torch

from oracle import oracle as O
from pearl_b200 import _lib
from pearl_b200 import merkle as MK

KEY = b"0123456789abcdef0123456789abcdef"  # merkle.rs test_key


def _data(size):
    return (np.arange(size) % 256).astype(np.uint8)  # merkle.rs test_data


def _padded(d):
    return d.tobytes().ljust(MK.padded_chunk_len(d.size), b"\0")


@pytest.mark.parametrize("size", [1, 100, 1023, 1024, 1025, 2000, 3000, 7777, 2 * 1024, 3 * 1024, 5 * 1024,
                                  7 * 1024, 10 * 1024, 129 * 1024 + 3])
def test_oracle_root_is_keyed_blake3_of_padded_bytes(size):
    """merkle.rs test_root_matches_blake3_hash / _partial_last_chunk, on the
    zero-padded bytes the miner hashes (matrix_merkle_tree.py:26,44-47)."""
    blake3 = pytest.importorskip("blake3")
    d = _data(size)
    layers = O.merkle_layers(d, KEY)
    assert layers[-1][0].tobytes() == blake3.blake3(_padded(d), key=KEY).digest()
    assert layers[-1][0].tobytes() == O.tensor_hash(d, KEY)
    assert [len(x) for x in layers] == MK.merkle_layer_sizes(size)


def test_layer_sizes_match_library():
    L = _lib.load()
    for size in [0, 1, 1024, 1025, 2048, 3072, 4096, 128 * 1024, 128 * 1024 + 1, 8192 * 8192, 940 * 2 ** 20]:
        assert L.pb2_merkle_nodes(size) == sum(MK.merkle_layer_sizes(size))


@pytest.mark.parametrize("indices", [[0], [2], [4], [7], [0, 1], [2, 3, 4], [0, 2], [0, 3], [1, 3, 5],
                                     [0, 1, 4, 5], [0, 2, 3, 7], list(range(8))])
def test_proof_round_trip_8_leaves(indices):
    """merkle.rs test_single_leaf_proof / _consecutive / _non_consecutive /
    test_full_tree_proof; the host walk equals the oracle's."""
    d = _data(8 * 1024)
    layers = O.merkle_layers(d, KEY)
    want = O.multileaf_proof(layers, d.tobytes(), indices)
    got = MK.multileaf_proof(layers, indices, lambda i: d.tobytes()[i * 1024:(i + 1) * 1024])
    assert got.siblings == want["siblings"] and got.leaf_indices == want["leaf_indices"]
    assert got.leaf_data == want["leaf_data"] and got.root == want["root"] and got.total_leaves == 8
    assert O.proof_root(want, KEY) == want["root"]
    if len(indices) == 8:
        assert got.siblings == []


def test_proof_lengths_dedup_and_rejection():
    """merkle.rs test_4_leaf_proof_lengths, test_proof_dedup_and_ordering and
    the test_reject_* cases."""
    d4 = _data(4 * 1024)
    l4 = O.merkle_layers(d4, KEY)
    lens = [len(MK.multileaf_proof(l4, i, lambda _: b"").siblings) for i in ([0, 1], [0, 2], [0, 1, 2, 3])]
    assert lens == [1, 2, 0]
    d = _data(8 * 1024)
    layers = O.merkle_layers(d, KEY)
    chunk = lambda i: d.tobytes()[i * 1024:(i + 1) * 1024]  # noqa: E731
    assert MK.multileaf_proof(layers, [5, 3, 4, 3], chunk).siblings == \
        MK.multileaf_proof(layers, [3, 4, 5], chunk).siblings
    good = O.multileaf_proof(layers, d.tobytes(), [2, 3])
    bad = dict(good, leaf_data=[b"\xff" * 1024] + good["leaf_data"][1:])
    assert O.proof_root(bad, KEY) != good["root"]
    bad = dict(good, leaf_indices=[3, 4])
    assert O.proof_root(bad, KEY) != good["root"]
    extra = O.multileaf_proof(layers, d.tobytes(), [0, 2, 5])
    extra["siblings"] = extra["siblings"] + [b"\xbb" * 32]
    assert O.proof_root(extra, KEY) is None
    with pytest.raises(ValueError):
        MK.multileaf_proof(layers, [], chunk)
    with pytest.raises(ValueError):
        MK.multileaf_proof(layers, [8], chunk)


def test_random_round_trips():
    """merkle.rs test_random_round_trips: 3..22 leaves, random subsets."""
    rng = random.Random(5)
    for seed in range(20):
        n = 3 + seed % 20
        d = _data(n * 1024)
        layers = O.merkle_layers(d, KEY)
        idx = sorted(rng.sample(range(n), 1 + seed % n))
        got = MK.multileaf_proof(layers, idx, lambda i: d.tobytes()[i * 1024:(i + 1) * 1024])
        pr = {"leaf_data": got.leaf_data, "leaf_indices": got.leaf_indices, "total_leaves": got.total_leaves,
              "root": got.root, "siblings": got.siblings}
        assert O.proof_root(pr, KEY) == layers[-1][0].tobytes()


def test_leaf_indices_from_rows():
    """merkle.rs test_leaf_indices_from_rows."""
    f = MK.MerkleTree.compute_leaf_indices_from_rows
    assert f([0, 2], (4, 1024)) == [0, 2]
    assert f([0, 2], (4, 512)) == [0, 1]
    assert f([0], (2, 1500)) == [0, 1]


def test_matrix_tree_argument_errors():
    """matrix_merkle_tree.py:15-23 and its tests: checked before any GPU work."""
    with pytest.raises(ValueError, match="tensor must be non-empty"):
        MK.MatrixMerkleTree(torch.empty((0, 1024), dtype=torch.int8), KEY)
    with pytest.raises(ValueError, match="Expected 2D tensor"):
        MK.MatrixMerkleTree(torch.zeros((2, 2, 2), dtype=torch.int8), KEY)
    with pytest.raises(ValueError, match="Expected int8 tensor"):
        MK.MatrixMerkleTree(torch.zeros((2, 2), dtype=torch.float32), KEY)
    with pytest.raises(ValueError, match="Expected 32-byte key"):
        MK.MatrixMerkleTree(torch.zeros((2, 2), dtype=torch.int8), b"short")
    assert MK.padded_chunk_len(0) == 0 and MK.padded_chunk_len(1) == 1024 and MK.padded_chunk_len(1025) == 2048
