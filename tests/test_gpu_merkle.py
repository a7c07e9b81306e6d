"""Merkle layers built on the GPU (pb2_merkle_layers) against the oracle
restatement of pearl-blake3/src/merkle.rs, bit-exact, and proofs of a hit
tile's rows checked by rebuilding the root from them."""
import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O
from pearl_b200 import merkle as MK

pytestmark = pytest.mark.gpu

KEY = bytes(range(7, 39))


@pytest.mark.parametrize("size", [1, 100, 1024, 1025, 3000, 7777, 8 * 1024, 127 * 1024, 128 * 1024,
                                  128 * 1024 + 1, 130 * 1024 + 5, 256 * 1024, 257 * 1024, 300 * 1024,
                                  1000 * 1024 + 17, 4099 * 1024])
def test_layers_bit_exact(size):
    g = torch.Generator().manual_seed(size)
    host = torch.randint(0, 256, (size,), generator=g, dtype=torch.uint8)
    tree = MK.MerkleTree(host.cuda(), KEY)
    want = O.merkle_layers(host.numpy(), KEY)
    got = tree._layers()
    assert [len(x) for x in got] == [len(x) for x in want]
    for lw, lg in zip(want, got):
        assert np.array_equal(lw, lg)
    assert tree.root == O.tensor_hash(host.numpy(), KEY)


def test_hit_tile_proofs_8192():
    """A hit tile's A rows (rows r and r + 8 of the 2 x 64 tile pattern) and
    B rows (its 64 columns in B's (N, K) storage) at 8192 x 8192: the root is
    tensor_hash's and every proof rebuilds it."""
    g = torch.Generator().manual_seed(11)
    A = torch.randint(-64, 64, (8192, 8192), generator=g, dtype=torch.int8).cuda()
    key_t = torch.frombuffer(bytearray(KEY), dtype=torch.uint8).cuda()
    out = torch.empty(32, dtype=torch.uint8, device="cuda")
    roots = torch.empty(pg.get_required_scratchpad_bytes(A.numel(), 128), dtype=torch.uint8, device="cuda")
    pg.tensor_hash(A, key_t, out, roots, 128)
    tree = MK.MatrixMerkleTree(A, KEY)
    assert tree.root == bytes(out.cpu().numpy())
    for rows in ([16, 24], [8176, 8184], list(range(4096, 4096 + 256, 4)), [0]):
        proof = tree.get_multileaf_proof(tree.leaf_indices_from_rows(rows))
        pr = {"leaf_data": proof.leaf_data, "leaf_indices": proof.leaf_indices,
              "total_leaves": proof.total_leaves, "root": proof.root, "siblings": proof.siblings}
        assert O.proof_root(pr, KEY) == tree.root
        assert proof.total_leaves == 65536
        for i, d in zip(proof.leaf_indices, proof.leaf_data):
            assert d == A.view(-1)[i * 1024:(i + 1) * 1024].cpu().numpy().tobytes()
    p2 = MK.open_rows(A, KEY, [16, 24])
    assert p2.siblings == tree.get_multileaf_proof(tree.leaf_indices_from_rows([16, 24])).siblings


def test_matrix_tree_leaves():
    """miner-base test_tensor_tiling_correctness: a changed row changes only
    its own leaf."""
    t1 = torch.zeros((2, 1024), dtype=torch.int8)
    t2 = torch.zeros((2, 1024), dtype=torch.int8)
    t1[0, :] = 1
    t2[0, :] = 2
    a = MK.MatrixMerkleTree(t1.cuda(), KEY).leaf_hashes
    b = MK.MatrixMerkleTree(t2.cuda(), KEY).leaf_hashes
    assert len(a) == 2 and a[0] != b[0] and a[1] == b[1]


def test_moe_routing_proof():
    """The routing proof of a hit in expert 3's slice: the opened chunks hold
    the routed tokens at the global rows, and the proof rebuilds the root of
    the routing data's tree (the routing_root of the MoE commitment)."""
    from pearl_b200 import moe
    g = torch.Generator().manual_seed(4)
    tokens, top_k, E = 3000, 2, 8
    ids = torch.stack([torch.randperm(E, generator=g)[:top_k] for _ in range(tokens)]).to(torch.int32).cuda()
    n = tokens * top_k
    rd = torch.empty(n, dtype=torch.int32, device="cuda")
    si = torch.empty(n, dtype=torch.int32, device="cuda")
    off = torch.empty(E, dtype=torch.int32, device="cuda")
    scratch = torch.empty(moe.get_build_routing_data_scratchpad_bytes(n), dtype=torch.uint8, device="cuda")
    moe.build_routing_data(ids, rd, si, off, scratch, E)
    offs = off.tolist()
    inner = [0, 8, 300, offs[3] - offs[2] - 1]
    res = MK.moe_routing_proof(rd, offs, 3, inner, KEY, E, top_k)
    p = res.routing_proof
    pr = {"leaf_data": p.leaf_data, "leaf_indices": p.leaf_indices, "total_leaves": p.total_leaves,
          "root": p.root, "siblings": p.siblings}
    assert p.root == O.tensor_hash(rd.cpu().numpy(), KEY)
    assert O.proof_root(pr, KEY) == p.root
    data = {i: d for i, d in zip(p.leaf_indices, p.leaf_data)}
    host = rd.cpu().numpy()
    for r in inner:
        gr = offs[2] + r
        leaf, at = divmod(4 * gr, 1024)
        assert np.frombuffer(data[leaf][at:at + 4], np.int32)[0] == host[gr]
    assert (res.e, res.top_k, res.expert_idx, res.inner_a_rows) == (E, top_k, 3, inner)
