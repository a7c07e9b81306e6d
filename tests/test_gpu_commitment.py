"""GPU parity of the commitment inputs of a mined GEMM: tensor_hash (keyed
BLAKE3 Merkle root of a byte tensor) and commitment_hash_from_merkle_roots
(the noise-seed chain), called through the reference-shaped API (and so the
C ABI), compared bit-exactly with the CPU oracle, which is pinned to the
blake3 package and to the consensus seed vectors of zk-pow/src/api/seed.rs
(tests/golden/commitment.json)."""

import json
import os

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()


def _dev(b: bytes) -> torch.Tensor:
    return torch.frombuffer(bytearray(b), dtype=torch.uint8).cuda()


def _gpu_tensor_hash(data: torch.Tensor, key: bytes, tpb: int = 128) -> bytes:
    out = torch.zeros(32, dtype=torch.uint8, device="cuda")
    roots = torch.full((pg.get_required_scratchpad_bytes(data.numel(), tpb),), 0xAB,
                       dtype=torch.uint8, device="cuda")
    pg.tensor_hash(data, _dev(key), out, roots, threads_per_block=tpb)
    return out.cpu().numpy().tobytes()


# Sizes straddle every boundary of the tree: a partial single chunk, one
# chunk, one group of 128 chunks, a group plus one chunk (an odd carry), many
# groups with a ragged tail, and large operands.
@pytest.mark.parametrize("rows,cols", [(1, 1), (1, 1000), (1, 1024), (1, 1040), (3, 1000),
                                       (128, 1024), (129, 1024), (300, 1000), (1024, 4096),
                                       (4099, 1312), (8192, 8192)])
def test_tensor_hash_matches_oracle(rows, cols):
    g = torch.Generator().manual_seed(rows * 7 + cols)
    data = torch.randint(0, 256, (rows, cols), generator=g, dtype=torch.uint8)
    key = bytes(np.random.default_rng(rows + cols).integers(0, 256, 32, dtype=np.uint8))
    want = O.tensor_hash(data.numpy(), key)
    assert _gpu_tensor_hash(data.cuda(), key) == want


# Ragged tails, exactly one group (the root applied inside the group), and
# whole groups only (every group on the staged-copy path).
@pytest.mark.parametrize("tpb,rows,cols", [(256, 777, 3000), (512, 777, 3000), (256, 256, 1024),
                                           (512, 512, 1024), (512, 1024, 2048), (256, 300, 1024)])
def test_tensor_hash_group_sizes(tpb, rows, cols):
    g = torch.Generator().manual_seed(tpb + rows)
    data = torch.randint(-128, 128, (rows, cols), generator=g, dtype=torch.int8)
    key = bytes(range(32))
    want = O.tensor_hash(data.numpy(), key)
    assert _gpu_tensor_hash(data.cuda().view(torch.uint8), key, tpb) == want


def test_tensor_hash_torch_op_and_validation():
    data = torch.arange(5000, dtype=torch.int32).to(torch.uint8).reshape(5, 1000).cuda()
    key = bytes(31 - i for i in range(32))
    out = torch.zeros(32, dtype=torch.uint8, device="cuda")
    roots = torch.empty(pg.get_required_scratchpad_bytes(data.numel()), dtype=torch.uint8,
                        device="cuda")
    torch.ops.pearl_gemm.tensor_hash(data, _dev(key), out, roots)
    assert out.cpu().numpy().tobytes() == O.tensor_hash(data.cpu().numpy(), key)
    with pytest.raises(RuntimeError, match="roots must have at least"):
        pg.tensor_hash(torch.zeros(300, 1024, dtype=torch.uint8, device="cuda"), _dev(key), out,
                       roots[:32])
    with pytest.raises(RuntimeError, match="threads_per_block"):
        pg.tensor_hash(data, _dev(key), out, roots, threads_per_block=64)


def _gpu_commitment(job_key, ha, hb, salted_dims=None, routing_root=None, offsets_hash=None):
    a = torch.zeros(32, dtype=torch.uint8, device="cuda")
    b = torch.zeros(32, dtype=torch.uint8, device="cuda")
    pg.commitment_hash_from_merkle_roots(
        _dev(ha), _dev(hb), _dev(job_key), a, b,
        None if routing_root is None else _dev(routing_root),
        None if offsets_hash is None else _dev(offsets_hash), salted_dims=salted_dims)
    return b.cpu().numpy().tobytes(), a.cpu().numpy().tobytes()


def _offsets_hash(offsets, job_key):
    # zk-pow/src/api/proof_utils.rs:34-45: keyed hash of the little-endian
    # u32 offsets zero-padded to 1 KiB chunks.
    return O.tensor_hash(np.asarray(offsets, dtype="<u4").view(np.uint8), job_key)


def test_commitment_consensus_vectors(golden_dir):
    g = json.load(open(os.path.join(golden_dir, "commitment.json")))
    jk, ha, hb = (bytes.fromhex(g[x]) for x in ("job_key", "hash_a", "hash_b"))
    for case in g["cases"]:
        dims = tuple(case["salted_dims"]) if case["salted_dims"] else None
        rr = bytes.fromhex(case["routing_root"]) if "routing_root" in case else None
        oh = _offsets_hash(case["offsets"], jk) if rr is not None else None
        b, a = _gpu_commitment(jk, ha, hb, dims, rr, oh)
        assert b.hex() == case["b_seed"] and a.hex() == case["a_seed"], case


@pytest.mark.parametrize("salted", [None, (8192, 28672), (1, 0xFFFFFFFF)])
@pytest.mark.parametrize("moe", [False, True])
def test_commitment_matches_oracle(salted, moe):
    rng = np.random.default_rng(11)
    jk, ha, hb, rr = (bytes(rng.integers(0, 256, 32, dtype=np.uint8)) for _ in range(4))
    offsets = [0, 130, 4096, 4097, 16384] if moe else None
    want = O.commitment(jk, ha, hb, salted_dims=salted, routing_root=rr if moe else None,
                        offsets=offsets)
    got = _gpu_commitment(jk, ha, hb, salted, rr if moe else None,
                          _offsets_hash(offsets, jk) if moe else None)
    assert got == want


def test_commitment_from_tensor_hashes_end_to_end():
    """The chain the mined layer runs (gemm_operators.py:111-150): roots of
    A and B on the GPU, then the seeds, equal to the oracle's whole chain."""
    g = torch.Generator().manual_seed(3)
    A = torch.randint(-64, 64, (512, 1024), generator=g, dtype=torch.int8)
    B = torch.randint(-64, 64, (768, 1024), generator=g, dtype=torch.int8)
    key = bytes(np.random.default_rng(9).integers(0, 256, 32, dtype=np.uint8))
    ra = torch.zeros(32, dtype=torch.uint8, device="cuda")
    rb = torch.zeros(32, dtype=torch.uint8, device="cuda")
    scratch = torch.empty(pg.get_required_scratchpad_bytes(768 * 1024), dtype=torch.uint8,
                          device="cuda")
    pg.tensor_hash(A.cuda().view(torch.uint8), _dev(key), ra, scratch)
    pg.tensor_hash(B.cuda().view(torch.uint8), _dev(key), rb, scratch)
    ca = torch.zeros(32, dtype=torch.uint8, device="cuda")
    cb = torch.zeros(32, dtype=torch.uint8, device="cuda")
    pg.commitment_hash_from_merkle_roots(ra, rb, _dev(key), ca, cb, salted_dims=(512, 768))
    want_b, want_a = O.commitment(key, O.tensor_hash(A.numpy(), key), O.tensor_hash(B.numpy(), key),
                                  salted_dims=(512, 768))
    assert cb.cpu().numpy().tobytes() == want_b and ca.cpu().numpy().tobytes() == want_a
