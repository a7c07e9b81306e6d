"""GPU parity of the mining layer of miner/vllm-miner on the B200 operators
(pearl_b200.miner): routing order, activation quantization, the dense mined
layer (pearl_gemm_noisy) and the MoE GEMM1 per-expert loop.  Integer
results (routing, commitment seeds, hit sets) are compared bit-exactly with
the CPU oracle; bf16 outputs within the reference's test tolerance
(test_pearl_gemm.py:720-728: atol 1e-1, rtol 1e-2)."""

import math

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O
from pearl_b200 import miner as MN

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


# ---------------------------------------------------------------- routing ---
@pytest.mark.parametrize("tokens,top_k,experts", [(96, 2, 4), (20000, 2, 8), (4096, 8, 256),
                                                  (1, 1, 1), (777, 3, 60)])
def test_build_routing_data_matches_stable_sort(tokens, top_k, experts):
    g = torch.Generator().manual_seed(tokens + experts)
    ids = torch.randint(0, max(1, experts - 1 if experts > 2 else experts), (tokens, top_k),
                        generator=g, dtype=torch.int32)  # leaves the last expert empty
    n = tokens * top_k
    rd = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    si = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    off = torch.full((experts,), -1, dtype=torch.int32, device="cuda")
    scratch = torch.empty(pg.moe.get_build_routing_data_scratchpad_bytes(n), dtype=torch.uint8,
                          device="cuda")
    torch.ops.pearl_gemm.build_routing_data(ids.cuda(), rd, si, off, scratch, experts)
    want_rd, want_si, want_off = O.routing_order(ids.numpy(), experts)
    assert np.array_equal(_np(si), want_si)
    assert np.array_equal(_np(rd), want_rd)
    assert np.array_equal(_np(off), want_off)


# --------------------------------------------------------------- quantize ---
def _ref_quant(x, smooth, max_val, block):
    """The reference's quantization (hadamard.py:443-517) restated in numpy
    float32, step for step: Sylvester butterflies with strides 1, 2, 4, ...
    (lower = a + b, upper = a - b), times fl(1/sqrt(k)), the first element
    of each block negated, times the smooth scale, amax of |v|, then
    inv = fl(max_val) * rcp.approx.ftz(amax + 1e-30) and
    q = clamp(rint(v * inv)), scale = amax * fl(1/max_val).  The approximate
    reciprocal is a hardware instruction whose last bit PTX leaves open, so
    it is read from the device (pg.quantization.rcp_approx_f32); every other
    step is plain IEEE float32 here."""
    v = x.float().numpy().astype(np.float32)
    if block:
        rows, n = v.shape
        b = v.reshape(rows, n // block, block).copy()
        s = 1
        while s < block:
            idx = np.arange(block)
            lo, hi = idx[(idx & s) == 0], idx[(idx & s) != 0]
            a_lo, a_hi = b[..., lo].copy(), b[..., hi].copy()
            b[..., lo] = a_lo + a_hi
            b[..., hi] = a_lo - a_hi
            s <<= 1
        b *= np.float32(1.0 / math.sqrt(block))
        b[..., 0] *= np.float32(-1)
        v = b.reshape(rows, n)
    if smooth is not None:
        v = v * smooth.numpy().astype(np.float32)
    amax = np.abs(v).max(1, keepdims=True).astype(np.float32)
    rcp = pg.quantization.rcp_approx_f32(torch.from_numpy(amax + np.float32(1e-30)).cuda()).cpu().numpy()
    inv = np.float32(max_val) * rcp
    q = np.clip(np.rint(v * inv), -max_val, max_val).astype(np.int8)
    return torch.from_numpy(q), torch.from_numpy(amax * np.float32(1.0 / max_val))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("block", [0, 16, 128])
@pytest.mark.parametrize("smooth", [None, "row", "per_token"])
def test_quantize_matches_reference_math(dtype, block, smooth):
    g = torch.Generator().manual_seed(block + (smooth is None))
    m, n = 300, 4096
    x = (torch.randn(m, n, generator=g) * 3).to(dtype)
    s = None
    if smooth == "row":
        s = torch.rand(1, n, generator=g) + 0.5
    elif smooth == "per_token":
        s = torch.rand(m, n, generator=g) + 0.5
    xq = torch.empty(m, n, dtype=torch.int8, device="cuda")
    xs = torch.empty(m, 1, dtype=torch.float32, device="cuda")
    pg.quantization.quantize(x.cuda(), xq, xs, smooth_scale=None if s is None else s.cuda(),
                             max_val=63, block_size=block)
    q_ref, s_ref = _ref_quant(x, s, 63, block)
    assert torch.equal(xq.cpu(), q_ref)
    assert torch.equal(xs.cpu(), s_ref)


@pytest.mark.parametrize("n", [8, 1024, 2056, 4096, 8192, 14336, 16384, 20480])
@pytest.mark.parametrize("block", [0, 128])
def test_quantize_row_lengths(n, block):
    """Every row-length class of the kernel (the row kept in registers for up
    to 1, 2, 4 or 8 vectors per thread, two passes over memory beyond)."""
    if block and n % block:
        pytest.skip("block must divide the row")
    g = torch.Generator().manual_seed(n + block)
    m = 64
    x = (torch.randn(m, n, generator=g) * 3).to(torch.bfloat16)
    xq = torch.empty(m, n, dtype=torch.int8, device="cuda")
    xs = torch.empty(m, 1, dtype=torch.float32, device="cuda")
    pg.quantization.quantize(x.cuda(), xq, xs, smooth_scale=None, max_val=63, block_size=block)
    q_ref, s_ref = _ref_quant(x, None, 63, block)
    assert torch.equal(xq.cpu(), q_ref)
    assert torch.equal(xs.cpu(), s_ref)


# ------------------------------------------------------------ dense layer ---
def _job(seed, frac=0.02, salted=True):
    key = bytes(np.random.default_rng(seed).integers(0, 256, 32, dtype=np.uint8))
    return key, salted


def _hits(mined, m, n):
    f = mined.sync_fields()
    assert f["error"] == 0
    return {(int(h[0]), int(h[1])) for h in _np(mined.hits)[: f["hit_count"]]}


def _oracle_digest_target(ap, bp, r, key, frac):
    ref = O.mine_tiles(ap, bp, r, key, 0)
    vals = sorted(sum(int(w) << (32 * i) for i, w in enumerate(d)) for d in ref.digests)
    return vals[max(0, int(len(vals) * frac) - 1)]


@pytest.mark.parametrize("salted", [True, False])
def test_pearl_gemm_noisy_chain_matches_oracle(salted):
    m, n, k, r = 256, 512, 1024, 128
    g = torch.Generator().manual_seed(31)
    A = torch.randint(-64, 64, (m, k), generator=g, dtype=torch.int8)
    B = torch.randint(-64, 64, (n, k), generator=g, dtype=torch.int8)
    sa, sb = torch.rand(m, generator=g) / 64, torch.rand(n, generator=g) / 64
    key, _ = _job(5)
    # The oracle's whole chain: roots, seeds, noise, transcripts, digests.
    ra, rb = O.tensor_hash(A.numpy(), key), O.tensor_hash(B.numpy(), key)
    seed_b, seed_a = O.commitment(key, ra, rb, salted_dims=(m, n) if salted else None)
    prob = O.noisy_problem(A.numpy(), B.numpy(), seed_a, seed_b, r)
    target = _oracle_digest_target(prob.ApEA, prob.BpEB, r, seed_a, 0.02)
    want = O.hit_set(O.mine_tiles(prob.ApEA, prob.BpEB, r, seed_a, target), m, n)
    hits = torch.zeros(4 * len(want) + 16, 12, dtype=torch.uint32, device="cuda")
    C, mined = MN.pearl_gemm_noisy(A.cuda(), B.cuda(), sa.cuda(), sb.cuda(), torch.bfloat16,
                                   MN.MiningJob(key, target, salted), hits=hits)
    torch.cuda.synchronize()
    assert _np(mined.commitment_hash_A).tobytes() == seed_a
    assert _np(mined.commitment_hash_B).tobytes() == seed_b
    assert _hits(mined, m, n) == want
    ref = (A.float() @ B.float().T) * sa[:, None] * sb[None, :]
    torch.testing.assert_close(C.float().cpu(), ref.to(torch.bfloat16).float(), atol=ATOL, rtol=RTOL)
    MN.release_header(mined.host_signal_header_pinned)


def test_pearl_linear_apply_weights_branches():
    class Layer:
        pass

    g = torch.Generator().manual_seed(8)
    m, n, k = 384, 512, 1024
    layer = Layer()
    layer.weight = torch.randint(-63, 64, (n, k), generator=g, dtype=torch.int8).cuda()
    layer.weight_scale = (torch.rand(n, 1, generator=g) / 64).cuda()
    layer.smooth_quant_scale = (torch.rand(k, generator=g) + 0.5).cuda()
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    cfg = MN.MiningConfig(min_m=256, min_n=256, min_k=256)
    key, _ = _job(6)
    lin = MN.PearlLinear(True, cfg, MN.MiningJob(key, 0, True))
    y_mined = lin.apply_weights(layer, x)
    assert len(lin.mined) == 1 and lin.mined[0].sync_fields()["error"] == 0
    xq, xs, _ = MN.quant_7bit(x, layer.smooth_quant_scale)
    ref = (xq.float() @ layer.weight.float().T) * xs * layer.weight_scale.reshape(1, -1)
    torch.testing.assert_close(y_mined.float(), ref.to(torch.bfloat16).float(), atol=ATOL, rtol=RTOL)
    small = MN.PearlLinear(True, MN.MiningConfig(), MN.MiningJob(key, 0, True))  # below thresholds
    torch.testing.assert_close(small.apply_weights(layer, x).float(), y_mined.float(), atol=ATOL,
                               rtol=RTOL)
    assert not small.mined
    y8 = MN.PearlLinear(False).apply_weights(layer, x)
    xq8, xs8, _ = MN.quant_8bit(x, layer.smooth_quant_scale)
    ref8 = (xq8.float() @ layer.weight.float().T) * xs8 * layer.weight_scale.reshape(1, -1)
    torch.testing.assert_close(y8.float(), ref8.to(torch.bfloat16).float(), atol=ATOL, rtol=RTOL)


def test_weight_root_cached_per_job_and_refreshed_after_a_write():
    """A layer's weight is hashed once per job: a second GEMM of the same
    weight reuses the root (same commitment seeds as a fresh hash, from the
    oracle), and an in-place write to the weight makes the next GEMM hash
    it again."""
    class Layer:
        pass

    g = torch.Generator().manual_seed(18)
    m, n, k = 384, 512, 1024
    layer = Layer()
    layer.weight = torch.randint(-63, 64, (n, k), generator=g, dtype=torch.int8).cuda()
    layer.weight_scale = (torch.rand(n, 1, generator=g) / 64).cuda()
    cfg = MN.MiningConfig(min_m=256, min_n=256, min_k=256)
    key, _ = _job(16)
    job = MN.MiningJob(key, 0, True)
    lin = MN.PearlLinear(True, cfg, job)
    for i in range(3):
        if i == 2:
            layer.weight.add_(1)  # a new version of the weight
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
        lin.apply_weights(layer, x)
        torch.cuda.synchronize()
        xq, _, _ = MN.quant_7bit(x)
        ra = O.tensor_hash(_np(xq), key)
        rb = O.tensor_hash(_np(layer.weight), key)
        seed_b, seed_a = O.commitment(key, ra, rb, salted_dims=(m, n))
        assert _np(lin.mined[-1].commitment_hash_B).tobytes() == seed_b, i
        assert _np(lin.mined[-1].commitment_hash_A).tobytes() == seed_a, i
    assert len({id(v[1]) for v in MN._B_ROOTS.values()}) >= 2
    for mnd in lin.mined:
        MN.release_header(mnd.host_signal_header_pinned)


# -------------------------------------------------------------- MoE GEMM1 ---
@pytest.mark.parametrize("grouped", [True, False])
def test_moe_gemm1_per_expert_parity(grouped):
    E, tokens, top_k, N, K, r = 4, 200, 2, 256, 512, 128
    g = torch.Generator().manual_seed(12)
    A = torch.randint(-64, 64, (tokens, K), generator=g, dtype=torch.int8)
    sa = torch.rand(tokens, 1, generator=g) / 64
    w1 = torch.randint(-64, 64, (E, N, K), generator=g, dtype=torch.int8)
    w1s = torch.rand(E, N, generator=g) / 64
    ids = torch.stack([torch.randperm(E, generator=g)[:top_k] for _ in range(tokens)]).to(torch.int32)
    key, _ = _job(13)
    target = 1 << 251  # ~1 in 32 full hash tiles
    out, res = MN.moe_gemm1(A.cuda(), sa.cuda(), ids.cuda(), w1.cuda(), w1s.cuda(),
                            MN.MiningJob(key, target, True), hit_capacity=4096, grouped=grouped)
    torch.cuda.synchronize()
    # Commitment: roots of A and the stacked weights, routing order and offsets.
    rd, si, off = O.routing_order(ids.numpy(), E)
    assert np.array_equal(_np(res.ctx.routing_data), rd) and np.array_equal(_np(res.ctx.routing_layout.slot_indices), si)
    oh = O.tensor_hash(off.astype("<u4").view(np.uint8), key)
    assert _np(res.ctx.offsets_hash).tobytes() == oh
    rr = O.tensor_hash(rd.astype("<i4").view(np.uint8), key)
    seed_b, seed_a = O.commitment(key, O.tensor_hash(A.numpy(), key),
                                  O.tensor_hash(w1.reshape(E * N, K).numpy(), key),
                                  salted_dims=(tokens, N), routing_root=rr, offsets=off.tolist())
    assert _np(res.ctx.commitment_hash_A).tobytes() == seed_a
    assert _np(res.ctx.commitment_hash_B).tobytes() == seed_b
    # Each expert's mined GEMM: noise rows follow the routed tokens.
    EAL = O.noise_dense(seed_a, "A", tokens, r)
    EBR = O.noise_dense(seed_b, "B", E * N, r)
    EAR, EBL = O.noise_pairs(seed_a, "A", K, r), O.noise_pairs(seed_b, "B", K, r)
    total = 0
    for e in range(E):
        start = 0 if e == 0 else int(off[e - 1])
        cnt = int(off[e]) - start
        toks = rd[start:start + cnt]
        ap = O.noise_operand(A.numpy()[toks], EAL[toks], EAR)
        bp = O.noise_operand(w1[e].numpy(), EBR[e * N:(e + 1) * N], EBL)
        m16 = -(-cnt // 16) * 16
        ap16 = np.zeros((m16, K), np.int8)
        ap16[:cnt] = ap
        want = {h for h in O.hit_set(O.mine_tiles(ap16, bp, r, seed_a, target), m16, N)
                if h[0] + 8 < cnt}
        mined = res.per_expert[e]
        assert _hits(mined, cnt, N) == want, e
        total += len(want)
        ref = (A[toks].float() @ w1[e].float().T) * sa[toks] * w1s[e][None, :]
        got = out[torch.from_numpy(si[start:start + cnt]).long()].float().cpu()
        torch.testing.assert_close(got, ref.to(torch.bfloat16).float(), atol=ATOL, rtol=RTOL)
        MN.release_header(mined.host_signal_header_pinned)
    assert total > 0


@pytest.mark.gpu
def test_scatter_rows_matches_index_put():
    """The MoE layer's row scatter (pb2_scatter_rows) writes exactly what
    torch's dst[indices] = src writes, for bf16 rows of a MoE-sized width,
    with a permutation and with indices outside dst skipped."""
    from pearl_b200.moe import scatter_rows
    g = torch.Generator(device="cuda").manual_seed(3)
    rows, n = 1000, 28672
    src = torch.randn(rows, n, generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(1500, generator=g, device="cuda")[:rows].to(torch.int32)
    want = torch.zeros(1500, n, dtype=torch.bfloat16, device="cuda")
    want[perm.long()] = src
    got = torch.zeros_like(want)
    scatter_rows(src, got, perm)
    assert torch.equal(got, want)
    bad = perm.clone()
    bad[::7] = 5000  # outside dst: skipped
    got2 = torch.zeros_like(want)
    scatter_rows(src, got2, bad)
    keep = torch.ones(rows, dtype=torch.bool, device="cuda")
    keep[::7] = False
    want2 = torch.zeros_like(want)
    want2[perm[keep].long()] = src[keep]
    assert torch.equal(got2, want2)


# --------------------------------------------------------- pinned pool ---
def test_pinned_header_pool_contract():
    """acquire() hands out zeroed, distinct, 128-byte aligned pinned
    headers and blocks when all are out; release() zeroes a header and
    refuses one the pool did not hand out or that is already back."""
    import threading

    pool = pg.HostSignalHeaderPinnedPool(pool_size=3)
    bufs = [pool.acquire() for _ in range(3)]
    assert len({b.data_ptr() for b in bufs}) == 3
    for b in bufs:
        assert b.is_pinned() and b.dtype == torch.int8 and b.numel() == pg.get_host_signal_header_size()
        assert b.data_ptr() % 128 == 0 and int(b.abs().sum()) == 0
    bufs[0].fill_(7)
    got = []
    t = threading.Thread(target=lambda: got.append(pool.acquire()))
    t.start()
    t.join(0.2)
    assert t.is_alive() and not got  # every header is out: acquire waits
    pool.release(bufs[0])
    t.join(5)
    assert got and got[0].data_ptr() == bufs[0].data_ptr() and int(got[0].abs().sum()) == 0
    with pytest.raises(ValueError):
        pool.release(torch.zeros(pg.get_host_signal_header_size(), dtype=torch.int8, pin_memory=True))
    pool.release(bufs[1])
    with pytest.raises(ValueError):
        pool.release(bufs[1])
