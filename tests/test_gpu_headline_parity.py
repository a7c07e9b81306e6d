"""Bit-exact parity of the mined GEMM at the shapes the throughput numbers
are quoted on: every transcript, every digest and the hit set of the GPU
path against the CPU oracle (zk-pow/src/ffi/mine.rs:86-107 restated in
oracle/pearl_oracle.c), plus C against an exact int32 product.

* 8192 x 8192 x 8192, R = 128: the headline GEMM (524,288 hash tiles, 64
  folds per tile, seven rounds of tiles per 2-SM pair).
* 1024 x 4096 x 14336: the Llama-3-8B down projection (112 R-chunks, so
  seven folds land on every transcript word).
* 16384 x 8192 x 8192: the largest single-GPU GEMM of the nonce-sharded
  workload (1,048,576 hash tiles).

Each shape runs twice on the GPU: once with the debug outputs (every
transcript and digest written out) and once on the production path (hit
list and pinned header only), and both hit sets must equal the oracle's.
The target is the oracle's 1% digest quantile, so about 1% of the tiles hit.
"""

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O
from tests.gpu_problem import gen_noise, make_problem, run_noisy_gemm

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-1, 1e-2


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()


def _np(t):
    return t.cpu().numpy()


def _digest_ints(digests: np.ndarray) -> np.ndarray:
    """uint256 digests (8 little-endian words) as Python ints, for ordering."""
    return np.array([sum(int(w) << (32 * i) for i, w in enumerate(d)) for d in digests], dtype=object)


def _exact_c(p) -> torch.Tensor:
    """C = A_scales * (A . B^T) * B_scales with the product exact in int32
    (cuBLAS int8 GEMM, an implementation independent of the kernel under
    test), rounded to bf16 once."""
    ab = torch._int_mm(p.A, p.B.t())
    return (ab.float() * p.A_scales[:, None] * p.B_scales[None, :]).to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(8192, 8192, 8192), (1024, 4096, 14336), (16384, 8192, 8192)])
def test_mined_gemm_bit_exact_at_workload_shapes(m, n, k):
    r = 128
    p = make_problem(m, n, k, r, seed=(m + 3 * n + 7 * k) % 10007)
    gen_noise(p)
    o = O.noisy_problem(_np(p.A), _np(p.B), _np(p.key_a).tobytes(), _np(p.key_b).tobytes(), r)
    ref = O.mine_tiles(o.ApEA, o.BpEB, r, _np(p.key_a).tobytes(), 0)
    vals = _digest_ints(ref.digests)
    tiles = O.num_hash_tiles(m, n)
    target = int(np.sort(vals)[tiles // 100])
    want = {O.hash_tile_origin(m, n, int(t)) for t in np.nonzero(vals <= target)[0]}
    assert tiles // 200 < len(want) < tiles // 50

    tr = torch.zeros(tiles, 16, dtype=torch.uint32, device="cuda")
    dg = torch.zeros(tiles, 8, dtype=torch.uint32, device="cuda")
    hits = torch.zeros(len(want) + 64, 12, dtype=torch.uint32, device="cuda")
    header, sync = run_noisy_gemm(p, target, run_noising_B=True, transcripts=tr, digests=dg, hits=hits)
    torch.cuda.synchronize()
    f = pg.get_host_signal_sync_fields(sync)
    assert f["error"] == 0, f
    assert np.array_equal(_np(p.out["ApEA"]), o.ApEA)
    assert np.array_equal(_np(p.out["BpEB"]), o.BpEB)
    bad = np.nonzero((_np(tr) != ref.transcripts).any(1))[0]
    assert bad.size == 0, f"{bad.size} transcripts differ, first at tile {bad[:4]}"
    assert np.array_equal(_np(dg), ref.digests)
    assert f["hit_count"] == len(want)
    assert {(int(h[0]), int(h[1])) for h in _np(hits)[: f["hit_count"]]} == want
    hdr = pg.get_host_signal_header(header)
    assert int(hdr.status) == 1
    idx = pg.extract_indices(hdr)
    assert (idx.A_row_indices[0], idx.B_column_indices[0]) in want
    torch.testing.assert_close(p.out["C"].float(), _exact_c(p).float(), atol=ATOL, rtol=RTOL)

    # The production path: no debug outputs, the same hits.
    hits.zero_()
    _, sync = run_noisy_gemm(p, target, run_noising_B=True, hits=hits)
    torch.cuda.synchronize()
    f = pg.get_host_signal_sync_fields(sync)
    assert f["error"] == 0 and f["hit_count"] == len(want)
    assert {(int(h[0]), int(h[1])) for h in _np(hits)[: f["hit_count"]]} == want
