"""The timeout path of the bounded device-side waits, made to run out on
purpose without faulting anything: a wait on an mbarrier that nothing
completes, then the mined GEMM launched with a budget far shorter than its
operand loads.  Both must end on their own with PB2_ERR_DEVICE_TIMEOUT in
the error word, and the next regular call must give bit-exact results."""

import numpy as np
import pytest
import torch

import pearl_b200 as pg
from oracle import oracle as O
from pearl_b200 import _lib
from tests.gpu_problem import gen_noise, make_problem, run_noisy_gemm, signal_buffers

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    pg.device_waits.set_wait_budget_cycles(0)
    torch.cuda.synchronize()


def _np(t):
    return t.cpu().numpy()


def _check_regular_call(seed):
    """A small mined GEMM with the default budget, checked against the oracle."""
    m, n, k, r = 256, 512, 1024, 128
    p = make_problem(m, n, k, r, seed=seed)
    gen_noise(p)
    o = O.noisy_problem(_np(p.A), _np(p.B), _np(p.key_a).tobytes(), _np(p.key_b).tobytes(), r)
    ref = O.mine_tiles(o.ApEA, o.BpEB, r, _np(p.key_a).tobytes(), 0)
    tiles = O.num_hash_tiles(m, n)
    tr = torch.zeros(tiles, 16, dtype=torch.uint32, device="cuda")
    _, sync = run_noisy_gemm(p, 0, transcripts=tr)
    torch.cuda.synchronize()
    assert pg.get_host_signal_sync_fields(sync)["error"] == 0
    assert np.array_equal(_np(tr), ref.transcripts)


def test_wait_selftest_runs_out_and_returns():
    sync = torch.zeros(16, dtype=torch.int8, device="cuda")
    pg.device_waits.wait_selftest(sync, budget_cycles=1 << 18)
    torch.cuda.synchronize()
    assert pg.get_host_signal_sync_fields(sync)["error"] == _lib.PB2_ERR_DEVICE_TIMEOUT
    _check_regular_call(seed=71)


def test_wait_selftest_rejects_bad_budget():
    sync = torch.zeros(16, dtype=torch.int8, device="cuda")
    with pytest.raises(RuntimeError):
        pg.device_waits.wait_selftest(sync, budget_cycles=0)
    with pytest.raises(RuntimeError):
        pg.device_waits.wait_selftest(sync, budget_cycles=pg.device_waits.DEFAULT_WAIT_BUDGET_CYCLES + 1)


def test_mined_gemm_unwinds_when_its_waits_run_out():
    """With a 64-cycle budget a wait gives up: the abort reaches every role,
    the producer drains its loads, the MMA warp retires what it issued, TMEM
    is released, and the kernel returns with the timeout recorded.  A wait's
    first try_wait may sleep for a system-defined time before the budget is
    looked at, so the problem is long enough (K = 8192: 64 chunks per tile)
    that the hash warps' wait for a tile's transcripts outlasts it."""
    m, n, k, r = 512, 512, 8192, 128
    p = make_problem(m, n, k, r, seed=73)
    gen_noise(p)
    _, sync = run_noisy_gemm(p, 0)  # noised operands and factors in place
    torch.cuda.synchronize()
    assert pg.get_host_signal_sync_fields(sync)["error"] == 0
    prev = pg.device_waits.set_wait_budget_cycles(64)
    assert prev == pg.device_waits.DEFAULT_WAIT_BUDGET_CYCLES
    try:
        header, sync = signal_buffers()
        run_noisy_gemm(p, 0, header=header, sync=sync, run_noising_A=False, run_noising_B=False)
        torch.cuda.synchronize()
        assert pg.get_host_signal_sync_fields(sync)["error"] == _lib.PB2_ERR_DEVICE_TIMEOUT
    finally:
        assert pg.device_waits.set_wait_budget_cycles(0) == 64
    _check_regular_call(seed=74)
