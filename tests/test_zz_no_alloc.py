"""pb2_noisy_gemm_static_scratch: the mined GEMM for callers that cannot
allocate device memory (a host that only reaches the library through its C
ABI, or a process whose HBM belongs to another allocator's pool).  It keeps
the exact int32 noising projections in a fixed array inside the library
instead of the caller's AxEBL_int32 / EARxBpEB_int32 buffers.

The GPU test calls it through the C ABI twice in a row and checks each call
against pb2_noisy_gemm given caller-allocated int32 buffers on the same
inputs: the noised operands, half factors, every transcript and digest and
the hit set bit-exactly, C within the tolerance of the other GPU tests.  A
second call that saw the first call's leftovers in the shared array would
fail.  This file is collected last so that a run stopping at its first
failure has already run every other test."""

import ctypes

import numpy as np
import pytest
import torch

from pearl_b200 import _lib
from tests.gpu_problem import gen_noise, make_problem, signal_buffers

ATOL, RTOL = 1e-1, 1e-2


def _params(p, sync, header, target, key, hits, tr, dg, int32_factors):
    q = _lib.GemmParams()
    q.device = p.A.device.index if p.A.device.index is not None else torch.cuda.current_device()
    q.m, q.n, q.k, q.r = p.m, p.n, p.k, p.r
    for name in ("EAL", "EBR", "EAR_R_major", "EBL_R_major", "EAR_K_major", "EBL_K_major",
                 "EAL_fp16", "EBR_fp16"):
        setattr(q, name, p.noise[name].data_ptr())
    for name in ("ApEA", "BpEB", "AxEBL_fp16", "EARxBpEB_fp16", "C"):
        setattr(q, name, p.out[name].data_ptr())
    q.A, q.B = p.A.data_ptr(), p.B.data_ptr()
    q.A_scales, q.B_scales = p.A_scales.data_ptr(), p.B_scales.data_ptr()
    if int32_factors:
        q.AxEBL_int32 = p.out["AxEBL_int32"].data_ptr()
        q.EARxBpEB_int32 = p.out["EARxBpEB_int32"].data_ptr()
    q.host_signal_header_pinned, q.host_signal_sync = header.data_ptr(), sync.data_ptr()
    q.pow_target, q.pow_key = target.data_ptr(), key.data_ptr()
    q.tile_size_m, q.tile_size_n, q.tile_size_k = 128, 256, 128
    q.cluster_size_m = q.cluster_size_n = 1
    q.run_noising_a = q.run_noising_b = 1
    q.k_blocks_per_split_noising_a, q.k_blocks_per_split_noising_b = 2, 3
    q.hits, q.hit_capacity = hits.data_ptr(), hits.shape[0]
    q.transcripts, q.digests = tr.data_ptr(), dg.data_ptr()
    return q


def _run(entry, p, key_pair, target_value, int32_factors):
    """One mined GEMM through `entry` of the C ABI; returns every result."""
    import pearl_b200 as pg
    from oracle import oracle as O

    p.key_a.copy_(key_pair[0])
    p.key_b.copy_(key_pair[1])
    gen_noise(p)
    for t in p.out.values():
        t.zero_()
    header, sync = signal_buffers(p.A.device)
    tiles = O.num_hash_tiles(p.m, p.n)
    tr = torch.zeros(tiles, 16, dtype=torch.uint32, device=p.A.device)
    dg = torch.zeros(tiles, 8, dtype=torch.uint32, device=p.A.device)
    hits = torch.zeros(tiles, 12, dtype=torch.uint32, device=p.A.device)
    target = pg.make_pow_target_tensor(target_value, p.A.device)
    key = p.key_a.view(torch.uint32)
    q = _params(p, sync, header, target, key, hits, tr, dg, int32_factors)
    L = _lib.load()
    stream = torch.cuda.current_stream(p.A.device).cuda_stream
    _lib.check(getattr(L, entry)(ctypes.byref(q), ctypes.c_void_p(stream)), entry)
    torch.cuda.synchronize()
    f = pg.get_host_signal_sync_fields(sync)
    assert f["error"] == 0, f
    got = {k: p.out[k].cpu().clone() for k in ("ApEA", "BpEB", "AxEBL_fp16", "EARxBpEB_fp16", "C")}
    got["transcripts"], got["digests"] = tr.cpu(), dg.cpu()
    got["hits"] = {tuple(int(x) for x in h) for h in hits.cpu().numpy()[: f["hit_count"]]}
    got["hit_count"] = f["hit_count"]
    return got


@pytest.mark.gpu
def test_static_scratch_matches_caller_scratch_on_two_calls_in_a_row():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    m, n, k, r = 512, 768, 2048, 128
    p = make_problem(m, n, k, r, seed=77, int32_factors=True)
    g = torch.Generator().manual_seed(78)
    keys = [(torch.randint(0, 256, (32,), dtype=torch.uint8, generator=g).cuda(),
             torch.randint(0, 256, (32,), dtype=torch.uint8, generator=g).cuda()) for _ in range(2)]
    target = 1 << 251  # about one hash tile in 32 hits
    want = [_run("pb2_noisy_gemm", p, kp, target, int32_factors=True) for kp in keys]
    # Two calls in a row of the entry point that allocates nothing.
    got = [_run("pb2_noisy_gemm_static_scratch", p, kp, target, int32_factors=False) for kp in keys]
    for w, o in zip(want, got):
        for name in ("ApEA", "BpEB", "AxEBL_fp16", "EARxBpEB_fp16", "transcripts", "digests"):
            assert torch.equal(o[name], w[name]), name
        assert w["hit_count"] > 0
        assert o["hit_count"] == w["hit_count"] and o["hits"] == w["hits"]
        torch.testing.assert_close(o["C"].float(), w["C"].float(), atol=ATOL, rtol=RTOL)
    assert not torch.equal(got[0]["digests"], got[1]["digests"])  # the two calls differ


def test_static_scratch_rejects_oversize_and_caller_buffers():
    """Argument checks run before any CUDA call, so no GPU is needed."""
    L = _lib.load()
    q = _lib.GemmParams()
    q.m, q.n, q.k, q.r = 16384, 16384, 1024, 128
    q.run_noising_a = q.run_noising_b = 1
    st = L.pb2_noisy_gemm_static_scratch(ctypes.byref(q), None)
    assert st == _lib.PB2_ERR_SCRATCH_LIMIT
    assert b"static scratch" in L.pb2_status_string(st)
    q.m = q.n = 8192  # exactly the limit; now a caller buffer is the error
    q.AxEBL_int32 = 16
    assert L.pb2_noisy_gemm_static_scratch(ctypes.byref(q), None) == _lib.PB2_ERR_INVALID_ARGUMENT
    assert L.pb2_noisy_gemm_static_scratch(None, None) == _lib.PB2_ERR_INVALID_ARGUMENT
    assert np.int64(_lib.STATIC_SCRATCH_BYTES) == 8 * 1024 * 1024


def _complete_params():
    """Parameters that pass every argument check (placeholder addresses,
    16-byte aligned); nothing is launched with them."""
    q = _lib.GemmParams()
    q.m, q.n, q.k, q.r = 512, 512, 1024, 128
    for i, (name, _) in enumerate(_lib.GemmParams._fields_):
        if name in ("AxEBL_int32", "EARxBpEB_int32", "host_signal_header_pinned", "inner_hash_counter",
                    "hits", "transcripts", "digests"):
            continue
        if _ == ctypes.c_void_p:
            setattr(q, name, 0x10000 * (i + 1))
    q.tile_size_m, q.tile_size_n, q.tile_size_k = 128, 256, 128
    q.cluster_size_m = q.cluster_size_n = 1
    q.run_noising_a = q.run_noising_b = 1
    return q


@pytest.mark.parametrize("missing", ["A", "EAL", "EAR_R_major", "EBL_K_major", "B", "EBR", "EAR_K_major",
                                     "EBL_R_major", "ApEA", "C", "A_scales", "host_signal_sync",
                                     "pow_target", "EAL_fp16", "EARxBpEB_fp16"])
def test_static_scratch_rejects_missing_operands_before_any_cuda_call(missing):
    """A call with an absent operand returns PB2_ERR_INVALID_ARGUMENT before
    it selects the device or clears the shared array (no GPU here: any CUDA
    call would fail with PB2_ERR_CUDA instead), so a rejected call never
    disturbs a call still running on the array."""
    L = _lib.load()
    q = _complete_params()
    setattr(q, missing, None)
    assert L.pb2_noisy_gemm_static_scratch(ctypes.byref(q), None) == _lib.PB2_ERR_INVALID_ARGUMENT
    assert L.pb2_noisy_gemm(ctypes.byref(q), None) == _lib.PB2_ERR_INVALID_ARGUMENT
