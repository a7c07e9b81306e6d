"""PlainProof assembly (pearl_b200.proof; block_submission.py:14-88) from a
hit the GPU reported: the opened rows are the ones extract_indices reads
from the pinned header, the key is BLAKE3(header || mining configuration),
each Merkle proof rebuilds the oracle's tensor hash of its matrix under that
key, and the opened chunks hold the opened rows' bytes.  The MoE variant
carries the routing proof of the hit's expert segment."""

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O
from pearl_b200 import moe as pmoe
from pearl_b200 import proof as PF
from tests.gpu_problem import gen_noise, make_problem, run_noisy_gemm

pytestmark = pytest.mark.gpu

HEADER = bytes(range(80))            # stand-in incomplete block header
CONFIG = b"pearl-mining-config:" + bytes(range(44))  # stand-in serialized configuration


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()


def _check_matrix_proof(mp: PF.MatrixMerkleProof, T: torch.Tensor, rows, key: bytes):
    host = T.contiguous().cpu().numpy().reshape(-1).view(np.uint8)
    proof = mp.proof
    assert mp.row_indices == [int(r) for r in rows]
    assert proof.root == O.tensor_hash(host, key)
    pr = {"leaf_data": proof.leaf_data, "leaf_indices": proof.leaf_indices, "total_leaves": proof.total_leaves,
          "root": proof.root, "siblings": proof.siblings}
    assert O.proof_root(pr, key) == proof.root
    chunks = dict(zip(proof.leaf_indices, proof.leaf_data))
    width = T.shape[1]
    for r in rows:
        lo, hi = int(r) * width, (int(r) + 1) * width
        for c in range(lo // 1024, (hi - 1) // 1024 + 1):
            want = host[c * 1024:(c + 1) * 1024].tobytes()
            assert chunks[c][:len(want)] == want


def test_plain_proof_from_a_gpu_hit():
    m, n, k, r = 512, 768, 1024, 128
    p = make_problem(m, n, k, r, seed=91)
    gen_noise(p)
    header, sync = run_noisy_gemm(p, (1 << 256) - 1)  # every whole hash tile hits
    torch.cuda.synchronize()
    assert pg.get_host_signal_sync_fields(sync)["status"] == 1
    hdr = pg.get_host_signal_header(header)
    idx = pg.extract_indices(hdr)
    assert len(idx.A_row_indices) == 2 and len(idx.B_column_indices) == 64
    opened = PF.opened_block_from_hit(hdr, p.A, p.B, r)
    proof = PF.create_proof(opened, HEADER, CONFIG)
    key = O.blake3(HEADER + CONFIG)
    assert PF.commitment_key(HEADER, CONFIG) == key
    assert (proof.m, proof.n, proof.k, proof.noise_rank, proof.moe) == (m, n, k, r, None)
    _check_matrix_proof(proof.a_merkle_proof, p.A, idx.A_row_indices, key)
    _check_matrix_proof(proof.bt_merkle_proof, p.B, idx.B_column_indices, key)
    # The roots are the ones the commitment is built from (tensor_hash).
    same = PF.create_proof(opened, hash_key=key)
    assert same.a_merkle_proof.proof.siblings == proof.a_merkle_proof.proof.siblings


def test_moe_plain_proof_carries_the_routing_proof():
    g = torch.Generator().manual_seed(12)
    tokens, top_k, E, n_per, k = 1000, 2, 8, 256, 1024
    ids = torch.stack([torch.randperm(E, generator=g)[:top_k] for _ in range(tokens)]).to(torch.int32).cuda()
    nr = tokens * top_k
    rd = torch.empty(nr, dtype=torch.int32, device="cuda")
    si = torch.empty(nr, dtype=torch.int32, device="cuda")
    off = torch.empty(E, dtype=torch.int32, device="cuda")
    scratch = torch.empty(pmoe.get_build_routing_data_scratchpad_bytes(nr), dtype=torch.uint8, device="cuda")
    pmoe.build_routing_data(ids, rd, si, off, scratch, E)
    offs = off.tolist()
    e = 5
    rows_e = offs[e] - offs[e - 1]
    A = torch.randint(-64, 64, (rows_e, k), generator=g, dtype=torch.int8).cuda()  # the expert's A slice
    B_t = torch.randint(-64, 64, (E * n_per, k), generator=g, dtype=torch.int8).cuda()  # every expert stacked
    inner_rows, inner_cols = [3, 11], list(range(e * n_per + 64, e * n_per + 128))
    block = PF.MoEBlock(expert_index=e, num_experts=E, n_per_expert=n_per, top_k=top_k, inner_a_rows=inner_rows,
                        inner_b_cols=inner_cols, routing_data=rd, expert_routing_offsets=offs)
    opened = PF.OpenedBlock(A_row_indices=inner_rows, B_column_indices=inner_cols, A=A, B_t=B_t, noise_rank=128,
                            moe=block)
    key = O.blake3(HEADER + CONFIG)
    proof = PF.create_proof(opened, hash_key=key)
    assert (proof.m, proof.n, proof.k) == (rows_e, n_per, k)
    _check_matrix_proof(proof.a_merkle_proof, A, inner_rows, key)
    _check_matrix_proof(proof.bt_merkle_proof, B_t, inner_cols, key)
    want = pg.merkle.moe_routing_proof(rd, offs, e, inner_rows, key, E, top_k)
    got = proof.moe
    assert (got.e, got.top_k, got.expert_idx, got.routing_end_offsets, got.inner_a_rows) == \
        (E, top_k, e, offs, inner_rows)
    assert got.routing_proof.root == want.routing_proof.root == O.tensor_hash(rd.cpu().numpy(), key)
    assert got.routing_proof.siblings == want.routing_proof.siblings


def test_create_proof_rejects_bad_inputs():
    A = torch.zeros(4, 64, dtype=torch.int8, device="cuda")
    B_t = torch.zeros(8, 32, dtype=torch.int8, device="cuda")
    opened = PF.OpenedBlock([0], [0], A, B_t, 128)
    with pytest.raises(ValueError):
        PF.create_proof(opened, hash_key=bytes(32))  # k mismatch
    opened.B_t = torch.zeros(8, 64, dtype=torch.int8, device="cuda")
    with pytest.raises(ValueError):
        PF.create_proof(opened)  # no key material
    with pytest.raises(ValueError):
        PF.create_proof(opened, hash_key=bytes(31))
