"""The grouped mined GEMM (pb2_noisy_gemm_grouped): every expert's mined
GEMM of a MoE layer in one noising and one persistent launch must give what
one noisy_gemm per expert gives (the reference's loop,
miner/vllm-miner/src/vllm_miner/pearl_moe_experts.py:304-343): the same
noised operands, every transcript and digest, the same hits per expert, the
same sync words and C.  Expert sizes include an empty expert, sizes that
are not multiples of the 256-row tile (tiles that end inside an expert) and
a width that is not a multiple of 256."""

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from pearl_b200 import moe

pytestmark = pytest.mark.gpu



@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()


def _problem(counts, n, k, r, seed):
    g = torch.Generator().manual_seed(seed)
    E, m = len(counts), sum(counts)
    dev = "cuda"
    t = dict(
        A=torch.randint(-64, 64, (m, k), generator=g, dtype=torch.int8).to(dev),
        B=torch.randint(-64, 64, (E * n, k), generator=g, dtype=torch.int8).to(dev),
        A_scales=(torch.rand(m, generator=g) / 64).to(dev),
        B_scales=(torch.rand(E * n, generator=g) / 64).to(dev))
    e = lambda *s, dt=torch.int8: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
    noise = dict(EAL=e(m, r), EBR=e(E * n, r), EAR_R_major=e(k, r), EBL_R_major=e(k, r),
                 EAR_K_major=e(r, k), EBL_K_major=e(r, k), EAL_fp16=e(m, r, dt=torch.float16),
                 EBR_fp16=e(E * n, r, dt=torch.float16))
    key_a = torch.randint(0, 256, (32,), generator=g, dtype=torch.uint8).to(dev)
    key_b = torch.randint(0, 256, (32,), generator=g, dtype=torch.uint8).to(dev)
    pg.noise_gen(R=r, key_A=key_a, key_B=key_b, **noise)
    t.update(noise)
    t["pow_key"] = key_a.view(torch.uint32)
    return t


def _outs(m, n_rows, k, r, n):
    e = lambda *s, dt=torch.int8: torch.zeros(*s, dtype=dt, device="cuda")  # noqa: E731
    return dict(ApEA=e(m, k), BpEB=e(n_rows, k), AxEBL_fp16=e(m, r, dt=torch.float16),
                EARxBpEB_fp16=e(n_rows, r, dt=torch.float16), C=e(m, n, dt=torch.bfloat16))


@pytest.mark.parametrize("counts,n,k,r,dumps", [
    ([256, 0, 48, 512, 160], 512, 1024, 128, True),
    ([300, 0, 17, 129, 5, 1000], 384, 768, 128, False),
    ([64, 208, 0, 96], 256, 1024, 64, True)])
def test_grouped_matches_one_noisy_gemm_per_expert(counts, n, k, r, dumps):
    E, m = len(counts), sum(counts)
    t = _problem(counts, n, k, r, seed=sum(counts) + n)
    target = pg.make_pow_target_tensor(1 << 251)  # about one hash tile in 32 hits
    row0 = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(int)
    tiles = [(c // 2) * (n // 64) for c in counts]

    # One grouped call.
    go = _outs(m, E * n, k, r, n)
    g_sync = [torch.zeros(16, dtype=torch.int8, device="cuda") for _ in range(E)]
    g_hdr = [torch.zeros(640, dtype=torch.int8).pin_memory() for _ in range(E)]
    g_hits = [torch.zeros(max(tl, 1) + 8, 12, dtype=torch.uint32, device="cuda") for tl in tiles]
    g_tr = [torch.zeros(tl, 16, dtype=torch.uint32, device="cuda") for tl in tiles] if dumps else None
    g_dg = [torch.zeros(tl, 8, dtype=torch.uint32, device="cuda") for tl in tiles] if dumps else None
    moe.noisy_gemm_grouped(
        t["A"], t["B"], t["EAL"], t["EAL_fp16"], t["EBR"], t["EBR_fp16"], t["EAR_R_major"], t["EBL_R_major"],
        t["EAR_K_major"], t["EBL_K_major"], go["AxEBL_fp16"], go["EARxBpEB_fp16"], go["ApEA"], go["BpEB"],
        t["A_scales"], t["B_scales"], go["C"], counts, g_hdr, g_sync, target, t["pow_key"], hits=g_hits,
        transcripts=g_tr, digests=g_dg)
    torch.cuda.synchronize()

    # One noisy_gemm per expert on its slices.
    total_hits = 0
    for e in range(E):
        c = counts[e]
        if c == 0:
            assert pg.get_host_signal_sync_fields(g_sync[e]) == {"lock": 0, "status": 0, "hit_count": 0,
                                                                 "error": 0}
            continue
        a, b = slice(row0[e], row0[e] + c), slice(e * n, (e + 1) * n)
        o = _outs(c, n, k, r, n)
        sync = torch.zeros(16, dtype=torch.int8, device="cuda")
        hdr = torch.zeros(640, dtype=torch.int8).pin_memory()
        hits = torch.zeros(max(tiles[e], 1) + 8, 12, dtype=torch.uint32, device="cuda")
        tr = torch.zeros(tiles[e], 16, dtype=torch.uint32, device="cuda") if dumps else None
        dg = torch.zeros(tiles[e], 8, dtype=torch.uint32, device="cuda") if dumps else None
        pg.noisy_gemm(A=t["A"][a], B=t["B"][b], EAL=t["EAL"][a], EAL_fp16=t["EAL_fp16"][a], EBR=t["EBR"][b],
                      EBR_fp16=t["EBR_fp16"][b], EAR_R_major=t["EAR_R_major"], EBL_R_major=t["EBL_R_major"],
                      EAR_K_major=t["EAR_K_major"], EBL_K_major=t["EBL_K_major"], A_scales=t["A_scales"][a],
                      B_scales=t["B_scales"][b], host_signal_header_pinned=hdr, host_signal_sync=sync,
                      pow_target=target, pow_key=t["pow_key"], hits=hits, transcripts=tr, digests=dg, **o)
        torch.cuda.synchronize()
        assert torch.equal(go["ApEA"][a], o["ApEA"]), e
        assert torch.equal(go["BpEB"][b], o["BpEB"]), e
        assert torch.equal(go["AxEBL_fp16"][a], o["AxEBL_fp16"]), e
        assert torch.equal(go["EARxBpEB_fp16"][b], o["EARxBpEB_fp16"]), e
        if dumps:
            assert torch.equal(g_tr[e], tr), e
            assert torch.equal(g_dg[e], dg), e
        f, gf = pg.get_host_signal_sync_fields(sync), pg.get_host_signal_sync_fields(g_sync[e])
        assert gf == f, (e, gf, f)
        got = {tuple(int(v) for v in h) for h in g_hits[e][: gf["hit_count"]].cpu().numpy()}
        want = {tuple(int(v) for v in h) for h in hits[: f["hit_count"]].cpu().numpy()}
        assert got == want, e
        total_hits += f["hit_count"]
        if f["hit_count"]:
            gh, hh = pg.get_host_signal_header(g_hdr[e]), pg.get_host_signal_header(hdr)
            gi = pg.extract_indices(gh)
            assert (gi.A_row_indices[0], gi.B_column_indices[0]) in {(int(h[0]), int(h[1])) for h in want}
            assert (gh.mma_size.m, gh.mma_size.n, gh.mma_size.k) == (hh.mma_size.m, hh.mma_size.n, hh.mma_size.k)
        assert torch.equal(go["C"][a], o["C"]), e  # the same MMAs in the same order
    assert total_hits > 0


def test_grouped_rejects_bad_expert_rows():
    counts = [64, 64]
    n, k, r = 256, 256, 128
    t = _problem(counts, n, k, r, seed=5)
    go = _outs(128, 2 * n, k, r, n)
    sync = [torch.zeros(16, dtype=torch.int8, device="cuda") for _ in counts]
    hdr = [None, None]
    args = (t["A"], t["B"], t["EAL"], t["EAL_fp16"], t["EBR"], t["EBR_fp16"], t["EAR_R_major"],
            t["EBL_R_major"], t["EAR_K_major"], t["EBL_K_major"], go["AxEBL_fp16"], go["EARxBpEB_fp16"],
            go["ApEA"], go["BpEB"], t["A_scales"], t["B_scales"], go["C"])
    target = pg.make_pow_target_tensor(0)
    with pytest.raises(RuntimeError):
        moe.noisy_gemm_grouped(*args, [64, 32], hdr, sync, target, t["pow_key"])  # rows do not add up
    with pytest.raises(RuntimeError):
        moe.noisy_gemm_grouped(*args, [64, 64], hdr[:1], sync[:1], target, t["pow_key"])


def test_grouped_row_map_writes_c_in_slot_order():
    """c_row_index fuses the slot-order write-back (pearl_moe_experts.py:347,
    cache_flat[idx] = out) into the epilogue: the destination gets exactly
    the rows the unmapped launch writes, moved by the index, and rows no
    index names are left alone; hits and sync words are unchanged."""
    counts, n, k, r = [300, 0, 17, 129, 5, 1000], 384, 768, 128
    E, m = len(counts), sum(counts)
    t = _problem(counts, n, k, r, seed=77)
    target = pg.make_pow_target_tensor(1 << 251)
    g = torch.Generator().manual_seed(5)
    idx = torch.randperm(m + 7, generator=g)[:m].to(torch.int32).cuda()

    def run(row_map):
        o = _outs(m, E * n, k, r, n)
        sync = [torch.zeros(16, dtype=torch.int8, device="cuda") for _ in range(E)]
        hdr = [torch.zeros(640, dtype=torch.int8).pin_memory() for _ in range(E)]
        dst = torch.full((m + 7, n), 3.0, dtype=torch.bfloat16, device="cuda") if row_map else o["C"]
        moe.noisy_gemm_grouped(
            t["A"], t["B"], t["EAL"], t["EAL_fp16"], t["EBR"], t["EBR_fp16"], t["EAR_R_major"],
            t["EBL_R_major"], t["EAR_K_major"], t["EBL_K_major"], o["AxEBL_fp16"], o["EARxBpEB_fp16"],
            o["ApEA"], o["BpEB"], t["A_scales"], t["B_scales"], dst, counts, hdr, sync, target, t["pow_key"],
            c_row_index=idx if row_map else None)
        torch.cuda.synchronize()
        return dst, [pg.get_host_signal_sync_fields(s) for s in sync]

    plain, f_plain = run(False)
    mapped, f_mapped = run(True)
    assert f_plain == f_mapped
    want = torch.full((m + 7, n), 3.0, dtype=torch.bfloat16, device="cuda")
    want[idx.long()] = plain
    assert torch.equal(mapped, want)
