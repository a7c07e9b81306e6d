"""The FP8 mined GEMM (pb2_mined_gemm_fp8), a builder-defined extension of the
mined contraction (the protocol has no FP8 mined GEMM).

* Integer-valued operands in [-8, 8] (exact in E4M3 and E5M2) keep every
  f32 partial sum exact, so the accumulation order does not matter: every
  transcript, digest and the hit set must then equal the CPU oracle's fold of
  the float32 bit patterns of the exact sums, and C the exact product.
* Normal(0, 1) operands with per-tensor scales: C within the tolerance below
  of the dequantized fp32 product, and two runs give identical transcripts
  (the f32 order is fixed by the kernel, not specified off the device)."""

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O

pytestmark = pytest.mark.gpu

# C of normal(0,1) FP8 operands: the f32 accumulation order differs from
# torch's, and C is rounded to bf16.
ATOL, RTOL = 5e-2, 1e-2


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()


def _buffers(m, n):
    tiles = (m // 2) * (n // 64)
    return dict(header=torch.zeros(640, dtype=torch.int8).pin_memory(),
                sync=torch.zeros(16, dtype=torch.int8, device="cuda"),
                hits=torch.zeros(tiles + 8, 12, dtype=torch.uint32, device="cuda"),
                tr=torch.zeros(tiles, 16, dtype=torch.uint32, device="cuda"),
                dg=torch.zeros(tiles, 8, dtype=torch.uint32, device="cuda"))


def _run(A8, B8, sa, sb, target, key, buf):
    m, n = A8.shape[0], B8.shape[0]
    C = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    pg.fp8.mined_gemm_fp8(A8, B8, sa, sb, C, buf["header"], buf["sync"], pg.make_pow_target_tensor(target), key,
                          hits=buf["hits"], transcripts=buf["tr"], digests=buf["dg"])
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("dtype", [torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("m,n,k", [(512, 768, 1024), (1024, 512, 4096)])
def test_fp8_transcripts_bit_exact_on_exact_sums(dtype, m, n, k):
    g = torch.Generator().manual_seed(m + k)
    Ai = torch.randint(-8, 9, (m, k), generator=g, dtype=torch.int8)
    Bi = torch.randint(-8, 9, (n, k), generator=g, dtype=torch.int8)
    key_b = np.random.default_rng(k).integers(0, 256, 32, dtype=np.uint8).tobytes()
    key = torch.frombuffer(bytearray(key_b), dtype=torch.uint8).cuda().view(torch.uint32)
    ref = O.mine_tiles(Ai.numpy(), Bi.numpy(), 128, key_b, 0, acc_f32=True)
    vals = sorted(sum(int(w) << (32 * i) for i, w in enumerate(d)) for d in ref.digests)
    target = vals[len(vals) // 50]
    want = O.hit_set(O.mine_tiles(Ai.numpy(), Bi.numpy(), 128, key_b, target, acc_f32=True), m, n)
    A8, B8 = Ai.float().to(dtype).cuda(), Bi.float().to(dtype).cuda()
    assert torch.equal(A8.float().cpu(), Ai.float())  # exactly representable
    one = torch.ones(1, dtype=torch.float32, device="cuda")
    buf = _buffers(m, n)
    C = _run(A8, B8, one, one, target, key, buf)
    assert np.array_equal(buf["tr"].cpu().numpy(), ref.transcripts)
    assert np.array_equal(buf["dg"].cpu().numpy(), ref.digests)
    f = pg.get_host_signal_sync_fields(buf["sync"])
    assert f["error"] == 0 and f["hit_count"] == len(want)
    assert {(int(h[0]), int(h[1])) for h in buf["hits"][: f["hit_count"]].cpu().numpy()} == want
    exact = (Ai.float() @ Bi.float().T).to(torch.bfloat16)
    assert torch.equal(C.cpu(), exact)


def test_fp8_normal_operands_within_tolerance_and_deterministic():
    m, n, k = 1024, 1536, 2048
    g = torch.Generator().manual_seed(5)
    Af = torch.randn(m, k, generator=g)
    Bf = torch.randn(n, k, generator=g)
    sa = torch.tensor([0.5], dtype=torch.float32, device="cuda")
    sb = torch.tensor([0.25], dtype=torch.float32, device="cuda")
    A8, B8 = Af.to(torch.float8_e4m3fn).cuda(), Bf.to(torch.float8_e4m3fn).cuda()
    key = torch.arange(8, dtype=torch.int32).to(torch.uint32).cuda()
    b1, b2 = _buffers(m, n), _buffers(m, n)
    C1 = _run(A8, B8, sa, sb, 1 << 251, key, b1)
    _run(A8, B8, sa, sb, 1 << 251, key, b2)
    assert torch.equal(b1["tr"], b2["tr"]) and torch.equal(b1["dg"], b2["dg"])
    ref = (A8.float() @ B8.float().T) * 0.5 * 0.25
    torch.testing.assert_close(C1.float(), ref.to(torch.bfloat16).float(), atol=ATOL, rtol=RTOL)
    f = pg.get_host_signal_sync_fields(b1["sync"])
    assert f["error"] == 0 and f["hit_count"] > 0


def test_fp8_rejects_mixed_formats():
    A8 = torch.zeros(256, 256, dtype=torch.float8_e4m3fn, device="cuda")
    B8 = torch.zeros(256, 256, dtype=torch.float8_e5m2, device="cuda")
    one = torch.ones(1, dtype=torch.float32, device="cuda")
    buf = _buffers(256, 256)
    with pytest.raises(RuntimeError):
        _run(A8, B8, one, one, 0, torch.zeros(8, dtype=torch.int32).to(torch.uint32).cuda(), buf)
