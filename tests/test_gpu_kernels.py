"""GPU parity tests: every kernel of the hot path, called through the
reference-shaped Python API (and so through the C ABI), compared with the
CPU oracle.  Integer outputs, transcripts, digests and hit sets must match
bit-exactly; the bf16 output C within the reference's own tolerance
(miner/pearl-gemm/tests/test_pearl_gemm.py:720-728: atol=1e-1, rtol=1e-2)."""

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O
from tests.gpu_problem import gen_noise, make_problem, run_noisy_gemm, signal_buffers

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


def oracle_problem(p):
    return O.noisy_problem(_np(p.A), _np(p.B), _np(p.key_a).tobytes(), _np(p.key_b).tobytes(), p.r)


def ref_c(p):
    ab = p.A.float().cpu() @ p.B.float().cpu().T  # exact in fp32 for these sizes
    return (ab * p.A_scales.cpu()[:, None] * p.B_scales.cpu()[None, :])


# ---------------------------------------------------------------- noise_gen
@pytest.mark.parametrize("m,n,k,r", [(256, 384, 512, 128), (192, 256, 320, 64), (1040, 256, 8192, 128)])
def test_noise_gen_bit_exact(m, n, k, r):
    p = make_problem(m, n, k, r, seed=m + k)
    gen_noise(p)
    o = oracle_problem(p)
    assert np.array_equal(_np(p.noise["EAL"]), o.EAL)
    assert np.array_equal(_np(p.noise["EBR"]), o.EBR)
    assert np.array_equal(_np(p.noise["EAR_R_major"]), O.pairs_to_r_major(o.EAR_pairs, r))
    assert np.array_equal(_np(p.noise["EBL_R_major"]), O.pairs_to_r_major(o.EBL_pairs, r))
    assert np.array_equal(_np(p.noise["EAR_K_major"]), O.pairs_to_r_major(o.EAR_pairs, r).T)
    assert np.array_equal(_np(p.noise["EBL_K_major"]), O.pairs_to_r_major(o.EBL_pairs, r).T)
    assert np.array_equal(_np(p.noise["EAL_fp16"]), (-1.0 * o.EAL).astype(np.float16))
    assert np.array_equal(_np(p.noise["EBR_fp16"]), (-4.0 * o.EBR).astype(np.float16))


def test_noise_gen_partial_outputs_and_aux():
    p = make_problem(128, 256, 256, 128, seed=3)
    aux = torch.full((1000,), 7, dtype=torch.int32, device="cuda")
    ear = torch.full((256, 128), 9, dtype=torch.int8, device="cuda")
    pg.noise_gen(R=128, EAR_R_major=ear, key_A=p.key_a, aux_buffer=aux)
    o = oracle_problem(p)
    assert np.array_equal(_np(ear), O.pairs_to_r_major(o.EAR_pairs, 128))
    assert int(aux.abs().sum()) == 0


# ------------------------------------------------------------ noise_A / B ---
@pytest.mark.parametrize("dtype", [torch.int32, torch.float16])
@pytest.mark.parametrize("m,k,r", [(256, 512, 128), (1025, 8192, 128), (128, 256, 64)])
def test_noise_A_bit_exact(m, k, r, dtype):
    p = make_problem(m, 256, k, r, seed=11)
    gen_noise(p)
    o = oracle_problem(p)
    axebl = torch.zeros(m, r, dtype=dtype, device="cuda")
    pg.noise_A(p.A, p.noise["EAL"], axebl, p.out["ApEA"], EAR=p.noise["EAR_R_major"],
               EBL=p.noise["EBL_K_major"])
    assert np.array_equal(_np(p.out["ApEA"]), o.ApEA)
    if dtype == torch.int32:
        assert np.array_equal(_np(axebl), o.AxEBL)
    else:
        want = (o.AxEBL.astype(np.float32) * 2.0 ** -14).astype(np.float16)
        assert np.array_equal(_np(axebl), want)


@pytest.mark.parametrize("dtype", [torch.int32, torch.float16])
@pytest.mark.parametrize("n,k,r", [(384, 512, 128), (1032, 4096, 128), (256, 320, 64)])
def test_noise_B_bit_exact(n, k, r, dtype):
    p = make_problem(128, n, k, r, seed=12)
    gen_noise(p)
    o = oracle_problem(p)
    proj = torch.zeros(n, r, dtype=dtype, device="cuda")
    pg.noise_B(p.B, p.noise["EBR"], proj, p.out["BpEB"], EAR=p.noise["EAR_K_major"],
               EBL=p.noise["EBL_R_major"])
    assert np.array_equal(_np(p.out["BpEB"]), o.BpEB)
    if dtype == torch.int32:
        assert np.array_equal(_np(proj), o.EARxBpEB)
    else:
        want = (o.EARxBpEB.astype(np.float32) * 2.0 ** -12).astype(np.float16)
        assert np.array_equal(_np(proj), want)


@pytest.mark.parametrize("dtype", [torch.float16, torch.int32])
@pytest.mark.parametrize("m,n,k,r", [(1025, 384, 1024, 128), (256, 2304, 4096, 128), (512, 512, 320, 64)])
def test_noise_AB_matches_noise_A_and_noise_B(m, n, k, r, dtype):
    """One launch for both operands (fp16 projections) or two (int32): the
    same bytes as the oracle's noise_A and noise_B."""
    p = make_problem(m, n, k, r, seed=13)
    gen_noise(p)
    o = oracle_problem(p)
    axebl = torch.zeros(m, r, dtype=dtype, device="cuda")
    earx = torch.zeros(n, r, dtype=dtype, device="cuda")
    pg.noise_AB(p.A, p.noise["EAL"], axebl, p.out["ApEA"], p.B, p.noise["EBR"], earx, p.out["BpEB"],
                **{k_: v for k_, v in p.noise.items() if k_ not in ("EAL", "EBR")})
    assert np.array_equal(_np(p.out["ApEA"]), o.ApEA)
    assert np.array_equal(_np(p.out["BpEB"]), o.BpEB)
    if dtype == torch.int32:
        assert np.array_equal(_np(axebl), o.AxEBL)
        assert np.array_equal(_np(earx), o.EARxBpEB)
    else:
        assert np.array_equal(_np(axebl), (o.AxEBL.astype(np.float32) * 2.0 ** -14).astype(np.float16))
        assert np.array_equal(_np(earx), (o.EARxBpEB.astype(np.float32) * 2.0 ** -12).astype(np.float16))


@pytest.mark.parametrize("m,n,k", [(8192, 8192, 1024), (16384, 8192, 512), (8000, 1000, 768)])
def test_noise_AB_row_blocks_below_256(m, n, k):
    """Large operands run with row blocks shorter than the 256-row MMA tile,
    so that every SM streams X (8192 + 8192 rows: 224-row blocks, the last
    one ragged; 16384 + 8192: 168-row blocks).  Rows of the tile past the
    block are computed and never stored: the outputs must still be the
    oracle's bytes."""
    p = make_problem(m, n, k, 128, seed=17)
    gen_noise(p)
    o = oracle_problem(p)
    axebl = torch.zeros(m, 128, dtype=torch.float16, device="cuda")
    earx = torch.zeros(n, 128, dtype=torch.float16, device="cuda")
    pg.noise_AB(p.A, p.noise["EAL"], axebl, p.out["ApEA"], p.B, p.noise["EBR"], earx, p.out["BpEB"],
                **{k_: v for k_, v in p.noise.items() if k_ not in ("EAL", "EBR")})
    assert np.array_equal(_np(p.out["ApEA"]), o.ApEA)
    assert np.array_equal(_np(p.out["BpEB"]), o.BpEB)
    assert np.array_equal(_np(axebl), (o.AxEBL.astype(np.float32) * 2.0 ** -14).astype(np.float16))
    assert np.array_equal(_np(earx), (o.EARxBpEB.astype(np.float32) * 2.0 ** -12).astype(np.float16))


def test_denoise_converter_bit_exact():
    g = torch.Generator().manual_seed(4)
    a = torch.randint(-30000, 30000, (512, 128), generator=g, dtype=torch.int32)
    b = torch.randint(-30000, 30000, (256, 128), generator=g, dtype=torch.int32)
    ao = torch.empty(512, 128, dtype=torch.float16, device="cuda")
    bo = torch.empty(256, 128, dtype=torch.float16, device="cuda")
    pg.denoise_converter(b.cuda(), a.cuda(), bo, ao)
    assert torch.equal(ao.cpu(), (a.float() * 2.0 ** -14).half())
    assert torch.equal(bo.cpu(), (b.float() * 2.0 ** -12).half())


# ------------------------------------------------------------- noisy_gemm ---
def _target_for_fraction(digests: np.ndarray, frac: float) -> int:
    vals = sorted(sum(int(w) << (32 * i) for i, w in enumerate(d)) for d in digests)
    return vals[max(0, int(len(vals) * frac) - 1)]


@pytest.mark.parametrize("m,n,k,r", [(1024, 1024, 1024, 128), (128, 256, 1024, 128),
                                     (256, 512, 2304, 64), (512, 768, 4096, 128)])
def test_noisy_gemm_transcripts_digests_hits_bit_exact(m, n, k, r):
    p = make_problem(m, n, k, r, seed=m + n + k)
    gen_noise(p)
    o = oracle_problem(p)
    ref = O.mine_tiles(o.ApEA, o.BpEB, r, _np(p.key_a).tobytes(), 0)
    target = _target_for_fraction(ref.digests, 0.01)
    ref_hits = O.hit_set(O.mine_tiles(o.ApEA, o.BpEB, r, _np(p.key_a).tobytes(), target), m, n)
    tiles = O.num_hash_tiles(m, n)
    tr = torch.zeros(tiles, 16, dtype=torch.uint32, device="cuda")
    dg = torch.zeros(tiles, 8, dtype=torch.uint32, device="cuda")
    hits = torch.zeros(4 * len(ref_hits) + 16, 12, dtype=torch.uint32, device="cuda")
    header, sync = run_noisy_gemm(p, target, transcripts=tr, digests=dg, hits=hits)
    torch.cuda.synchronize()
    assert np.array_equal(_np(p.out["ApEA"]), o.ApEA)
    assert np.array_equal(_np(p.out["BpEB"]), o.BpEB)
    assert np.array_equal(_np(tr), ref.transcripts)
    assert np.array_equal(_np(dg), ref.digests)
    f = pg.get_host_signal_sync_fields(sync)
    assert f["error"] == 0
    assert f["hit_count"] == len(ref_hits)
    got = {(int(h[0]), int(h[1])) for h in _np(hits)[: f["hit_count"]]}
    assert got == ref_hits
    hdr = pg.get_host_signal_header(header)
    assert int(hdr.status) == 1 and f["status"] == 1
    idx = pg.extract_indices(hdr)
    assert (idx.A_row_indices[0], idx.B_column_indices[0]) in ref_hits
    assert idx.A_row_indices[1] == idx.A_row_indices[0] + 8 and len(idx.B_column_indices) == 64
    torch.testing.assert_close(p.out["C"].float().cpu(), ref_c(p).to(torch.bfloat16).float(),
                               atol=ATOL, rtol=RTOL)


def test_noisy_gemm_golden_fixture(golden_dir):
    z = np.load(f"{golden_dir}/jackpot_m128_n256_k1024_r128.npz")
    m, k = z["A"].shape
    n = z["B"].shape[0]
    p = make_problem(m, n, k, 128, seed=0)
    p.A.copy_(torch.from_numpy(z["A"]))
    p.B.copy_(torch.from_numpy(z["B"]))
    p.key_a.copy_(torch.from_numpy(z["key_a"]))
    p.key_b.copy_(torch.from_numpy(z["key_b"]))
    gen_noise(p)
    tiles = O.num_hash_tiles(m, n)
    tr = torch.zeros(tiles, 16, dtype=torch.uint32, device="cuda")
    dg = torch.zeros(tiles, 8, dtype=torch.uint32, device="cuda")
    target = sum(int(w) << (32 * i) for i, w in enumerate(z["target"]))
    hits = torch.zeros(64, 12, dtype=torch.uint32, device="cuda")
    _, sync = run_noisy_gemm(p, target, transcripts=tr, digests=dg, hits=hits)
    torch.cuda.synchronize()
    assert np.array_equal(_np(tr), z["transcripts"])
    assert np.array_equal(_np(dg), z["digests"])
    f = pg.get_host_signal_sync_fields(sync)
    want = {O.hash_tile_origin(m, n, int(i)) for i in np.nonzero(z["hits"])[0]}
    assert {(int(h[0]), int(h[1])) for h in _np(hits)[: f["hit_count"]]} == want


@pytest.mark.parametrize("m,n,k", [(1025, 1032, 512), (128, 128, 256), (8192, 256, 256),
                                   (300, 6144, 1024)])
@pytest.mark.parametrize("scales", ["const", "variable"])
def test_noisy_gemm_output_within_tolerance(m, n, k, scales):
    p = make_problem(m, n, k, 128, seed=m * 3 + n, scales=scales)
    gen_noise(p)
    _, sync = run_noisy_gemm(p, 0)
    torch.testing.assert_close(p.out["C"].float().cpu(), ref_c(p).to(torch.bfloat16).float(),
                               atol=ATOL, rtol=RTOL)
    assert pg.get_host_signal_sync_fields(sync) == {"lock": 0, "status": 0, "hit_count": 0, "error": 0}


def test_noisy_gemm_int32_factors_and_split_k():
    p = make_problem(512, 512, 2048, 128, seed=21, int32_factors=True)
    gen_noise(p)
    o = oracle_problem(p)
    run_noisy_gemm(p, 0, k_blocks_per_split_noising_A=2, k_blocks_per_split_noising_B=3)
    assert np.array_equal(_np(p.out["AxEBL_int32"]), o.AxEBL)
    assert np.array_equal(_np(p.out["EARxBpEB_int32"]), o.EARxBpEB)
    torch.testing.assert_close(p.out["C"].float().cpu(), ref_c(p).to(torch.bfloat16).float(),
                               atol=ATOL, rtol=RTOL)


def test_many_rounds_per_cta_pair_bit_exact():
    """6144 x 6144 gives every 2-SM pair four rounds of tiles, so the
    transcript buffers of both slots are reused (the round-alternating
    buffers and the hash warps' clear-before-reuse); every transcript and
    digest must still match, and an all-pass target must hit every tile
    exactly once."""
    m = n = 6144
    k, r = 256, 128
    p = make_problem(m, n, k, r, seed=61)
    gen_noise(p)
    o = oracle_problem(p)
    ref = O.mine_tiles(o.ApEA, o.BpEB, r, _np(p.key_a).tobytes(), 0)
    tiles = O.num_hash_tiles(m, n)
    tr = torch.zeros(tiles, 16, dtype=torch.uint32, device="cuda")
    dg = torch.zeros(tiles, 8, dtype=torch.uint32, device="cuda")
    hits = torch.zeros(tiles + 8, 12, dtype=torch.uint32, device="cuda")
    _, sync = run_noisy_gemm(p, 2 ** 256 - 1, transcripts=tr, digests=dg, hits=hits)
    torch.cuda.synchronize()
    assert np.array_equal(_np(tr), ref.transcripts)
    assert np.array_equal(_np(dg), ref.digests)
    f = pg.get_host_signal_sync_fields(sync)
    assert f["error"] == 0 and f["hit_count"] == tiles
    got = {(int(h[0]), int(h[1])) for h in _np(hits)[:tiles]}
    assert len(got) == tiles


def test_all_tiles_hit_and_none_hit():
    m, n, k = 256, 512, 512
    p = make_problem(m, n, k, 128, seed=5)
    gen_noise(p)
    hits = torch.zeros(O.num_hash_tiles(m, n) + 8, 12, dtype=torch.uint32, device="cuda")
    _, sync = run_noisy_gemm(p, 2 ** 256 - 1, hits=hits)
    assert pg.get_host_signal_sync_fields(sync)["hit_count"] == O.num_hash_tiles(m, n)
    got = {(int(h[0]), int(h[1])) for h in _np(hits)[: O.num_hash_tiles(m, n)]}
    assert got == {O.hash_tile_origin(m, n, t) for t in range(O.num_hash_tiles(m, n))}
    _, sync = run_noisy_gemm(p, 0, hits=hits)
    assert pg.get_host_signal_sync_fields(sync)["hit_count"] == 0


def test_ragged_tiles_never_hit():
    # m, n not multiples of the hash-tile periods: partial tiles must not hit
    m, n, k = 200, 264, 256
    p = make_problem(m, n, k, 128, seed=6)
    gen_noise(p)
    hits = torch.zeros(4096, 12, dtype=torch.uint32, device="cuda")
    _, sync = run_noisy_gemm(p, 2 ** 256 - 1, hits=hits)
    f = pg.get_host_signal_sync_fields(sync)
    full_rows = sum(1 for r0 in range(m) if r0 % 16 < 8 and r0 + 8 < m)
    full_cols = sum(1 for c0 in range(0, n, 2) if (c0 % 256) < 8 and c0 + 249 < n)
    assert f["hit_count"] == full_rows * full_cols
    for h in _np(hits)[: f["hit_count"]]:
        assert h[0] + 8 < m and h[1] + 249 < n


def test_inner_hash_counter_formula():
    for m, n, k in [(512, 512, 256), (257, 512, 256), (1, 512, 256), (150, 504, 256)]:
        p = make_problem(max(m, 1), n, k, 128, seed=m)
        gen_noise(p)
        counter = torch.zeros(1, dtype=torch.int64, device="cuda")
        run_noisy_gemm(p, 0, run_noising_A=False, run_noising_B=False, inner_hash_counter=counter,
                       enable_debug=True)
        tiles = -(-m // 128) * -(-n // 256)
        assert int(counter.item()) == tiles * (k // 128) * (128 // 2) * (256 // 64)


@pytest.mark.parametrize("m,n,k", [
    (1000, 768, 1024),    # 128-wide tiles, one per SM pair
    (256, 4096, 4096),    # decode-batch shapes (Llama-3-8B o / qkv / gate_up / down): 128-wide tiles
    (256, 6144, 4096),
    (256, 28672, 4096),   # 224 narrow tiles: two per pair and round
    (256, 4096, 14336),
    (200, 1000, 384),     # ragged m and n
    (4096, 8192, 1024)])  # 256-wide tiles, two per pair and round
def test_gemm_vanilla(m, n, k):
    """The plain scaled GEMM (the vanilla branch of the mining layer) against
    an exact int32 product (cuBLAS int8, an implementation independent of
    the kernel), rounded to bf16 once."""
    g = torch.Generator().manual_seed(8 + m + n)
    A = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8).cuda()
    B = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).cuda()
    sa, sb = (torch.rand(m, generator=g) / 64).cuda(), (torch.rand(n, generator=g) / 64).cuda()
    C = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    pg.gemm(A, B, sa, sb, C)
    # _int_mm wants m > 16 and dims that are multiples of 8
    mp = -(-m // 8) * 8
    Ap = torch.zeros(mp, k, dtype=torch.int8, device="cuda")
    Ap[:m] = A
    np_ = -(-n // 8) * 8
    Bp = torch.zeros(np_, k, dtype=torch.int8, device="cuda")
    Bp[:n] = B
    ab = torch._int_mm(Ap, Bp.t())[:m, :n].float()
    ref = (ab * sa[:, None] * sb[None, :]).to(torch.bfloat16).float()
    torch.testing.assert_close(C.float(), ref, atol=ATOL, rtol=RTOL)


def test_torch_ops_schema_path():
    p = make_problem(256, 256, 512, 128, seed=9)
    gen_noise(p)
    header, sync = signal_buffers()
    torch.ops.pearl_gemm.noisy_gemm(
        p.A, p.B, p.noise["EAL"], p.noise["EAL_fp16"], p.noise["EBR"], p.noise["EBR_fp16"],
        p.noise["EAR_R_major"], p.noise["EBL_R_major"], p.noise["EAR_K_major"],
        p.noise["EBL_K_major"], p.out["AxEBL_fp16"], p.out["EARxBpEB_fp16"], p.out["ApEA"],
        p.out["BpEB"], p.A_scales, p.B_scales, p.out["C"], header, sync,
        pg.make_pow_target_tensor(0), p.key_a.view(torch.uint32), run_noising_B=True,
        skip_reduction=False)
    torch.testing.assert_close(p.out["C"].float().cpu(), ref_c(p).to(torch.bfloat16).float(),
                               atol=ATOL, rtol=RTOL)


def test_inner_hash_op():
    x = torch.arange(256, dtype=torch.int64).to(torch.uint32).cuda()
    want = 0
    for v in range(256):
        want ^= v
    assert int(pg.inner_hash(x, 1).item()) == want
    assert int(pg.inner_hash(x, 100000).item()) == (want * 100000) % 2 ** 32


def test_pearl_gemm_cuda_positional_calls():
    """The extension-module surface (pearl_b200.pearl_gemm_cuda) called the
    way the reference's pearl_gemm_interface.py calls its compiled extension:
    every argument positional, in the C++ order (pearl_gemm_api.cpp:168,
    618-656, 502-510).  Noise, noised operands and the hit set against the
    oracle, C within the reference tolerance."""
    from pearl_b200 import pearl_gemm_cuda as ext

    m, n, k, r = 256, 512, 1024, 128
    p = make_problem(m, n, k, r, seed=91)
    nz = p.noise
    ext.noise_gen(r, 64, nz["EAL"], nz["EAL_fp16"], nz["EAR_R_major"], nz["EAR_K_major"], nz["EBL_R_major"],
                  nz["EBL_K_major"], nz["EBR"], nz["EBR_fp16"], p.key_a, p.key_b, None)
    o = oracle_problem(p)
    assert np.array_equal(_np(nz["EAL"]), o.EAL) and np.array_equal(_np(nz["EBR"]), o.EBR)
    ref = O.mine_tiles(o.ApEA, o.BpEB, r, _np(p.key_a).tobytes(), 0)
    target = _target_for_fraction(ref.digests, 0.01)
    want = O.hit_set(O.mine_tiles(o.ApEA, o.BpEB, r, _np(p.key_a).tobytes(), target), m, n)
    header = torch.zeros(ext.get_host_signal_header_size(), dtype=torch.int8, pin_memory=True)
    sync = torch.zeros(ext.get_host_signal_sync_size(), dtype=torch.int8, device="cuda")
    out = p.out
    ext.noisy_gemm(p.A, p.B, nz["EAL"], nz["EAL_fp16"], nz["EBR"], nz["EBR_fp16"], nz["EAR_R_major"],
                   nz["EBL_R_major"], nz["EAR_K_major"], nz["EBL_K_major"], out["AxEBL_fp16"],
                   out["EARxBpEB_fp16"], out["ApEA"], out["BpEB"], p.A_scales, p.B_scales, out["C"], header, sync,
                   pg.make_pow_target_tensor(target), p.key_a.view(torch.uint32), None, None, 128, 256, 128, 1, 1,
                   None, None, True, None, None, None, None, 2, 2, None, None, True, True, False, False, None,
                   False)
    torch.cuda.synchronize()
    assert np.array_equal(_np(out["ApEA"]), o.ApEA) and np.array_equal(_np(out["BpEB"]), o.BpEB)
    f = pg.get_host_signal_sync_fields(sync)
    assert f["error"] == 0 and f["hit_count"] == len(want) and f["status"] == 1
    hdr = ext.get_host_signal_header(header)
    assert hdr.status == ext.HostSignalStatus.kSignalTriggered
    idx = pg.extract_indices(hdr)
    assert (idx.A_row_indices[0], idx.B_column_indices[0]) in want
    torch.testing.assert_close(out["C"].float().cpu(), ref_c(p).to(torch.bfloat16).float(), atol=ATOL, rtol=RTOL)
    C2 = torch.empty_like(out["C"])
    ext.gemm(p.A, p.B, p.A_scales, p.B_scales, C2, 128, 256, 128, 1, 1, None, None, True)
    torch.testing.assert_close(C2.float().cpu(), ref_c(p).to(torch.bfloat16).float(), atol=ATOL, rtol=RTOL)
