"""Split-K plain GEMM (pb2_gemm with a workspace): when few 256 x 256 tiles
cover C (decode batches), K is cut into equal ranges, each (tile, range)
work item writes its exact int32 partial and a second kernel sums and
scales.  The result must be the one the unsplit kernel gives, bit for bit,
and the exact int32 product scaled and rounded to bf16 once."""

import pytest
import torch

import pearl_b200 as pg
from pearl_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    torch.cuda.synchronize()


def _exact(A, B, sa, sb):
    m, n = A.shape[0], B.shape[0]
    mp, np_ = -(-max(m, 17) // 8) * 8, -(-n // 8) * 8
    Ap = torch.zeros(mp, A.shape[1], dtype=torch.int8, device="cuda")
    Ap[:m] = A
    Bp = torch.zeros(np_, B.shape[1], dtype=torch.int8, device="cuda")
    Bp[:n] = B
    ab = torch._int_mm(Ap, Bp.t())[:m, :n].float()
    return (ab * sa[:, None] * sb[None, :]).to(torch.bfloat16)


def _gemm(A, B, sa, sb, split: bool):
    C = torch.empty(A.shape[0], B.shape[0], dtype=torch.bfloat16, device="cuda")
    L = _lib.load()
    real = L.pb2_gemm_workspace_bytes
    if not split:
        L.pb2_gemm_workspace_bytes = lambda *args: 0
    try:
        pg.gemm(A, B, sa, sb, C)
    finally:
        L.pb2_gemm_workspace_bytes = real
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("m,n,k", [
    (256, 4096, 14336),   # Llama-3-8B down projection, decode batch (four ranges)
    (64, 4096, 14336),
    (200, 1000, 8192),    # ragged m and n (the last tile ends inside C)
    (1, 2048, 8192),      # one token
    (256, 2048, 6144)])   # the shortest split ranges (24 units)
def test_splitk_matches_unsplit_and_exact_product(m, n, k):
    assert _lib.load().pb2_gemm_workspace_bytes(0, m, n, k) > 0, "shape should take the split path"
    g = torch.Generator().manual_seed(m + n + k)
    A = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8).cuda()
    B = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).cuda()
    sa, sb = (torch.rand(m, generator=g) / 64).cuda(), (torch.rand(n, generator=g) / 64).cuda()
    C_split = _gemm(A, B, sa, sb, True)
    C_plain = _gemm(A, B, sa, sb, False)
    assert torch.equal(C_split, C_plain)
    assert torch.equal(C_split, _exact(A, B, sa, sb))


def test_no_split_for_large_problems():
    assert _lib.load().pb2_gemm_workspace_bytes(0, 8192, 8192, 8192) == 0
    assert _lib.load().pb2_gemm_workspace_bytes(0, 256, 28672, 4096) == 0  # 112 tiles fill the pairs
    assert _lib.load().pb2_gemm_workspace_bytes(0, 256, 4096, 256) == 0    # K too short to split
    assert _lib.load().pb2_gemm_workspace_bytes(0, 256, 4096, 4096) == 0   # ranges would be under 24 units
