"""Bounded device-side waits: the process-wide wait budget of the mined
GEMM's main kernel and a self-test of the timeout path (C ABI
pb2_set_wait_budget_cycles / pb2_wait_selftest).

Every wait inside these kernels (an mbarrier phase, a drain, a cluster
handshake) gives up after a budget of SM clock cycles: it records
PB2_ERR_DEVICE_TIMEOUT in the error word of the caller's host_signal_sync
buffer and the kernel unwinds and returns, so a stalled pipeline ends with a
status the host can read instead of holding the GPU.  The reference's
kernels have no such limit (their first-hit lock spins without one,
miner/pearl-gemm/csrc/gemm/pow_utils.hpp:267-269)."""

from __future__ import annotations

import torch

from . import _lib
from .pearl_gemm_interface import _device_index, _fail, _stream

DEFAULT_WAIT_BUDGET_CYCLES = _lib.DEFAULT_WAIT_BUDGET_CYCLES


def set_wait_budget_cycles(cycles: int) -> int:
    """Budget (SM cycles) that later launches of the mined GEMM's main kernel
    take, for the whole process; ``cycles <= 0`` restores the default (about
    one second).  Returns the previous budget.  Meant for tests and
    diagnostics: a budget shorter than a kernel's legitimate waits makes
    every launch end early with PB2_ERR_DEVICE_TIMEOUT."""
    return int(_lib.load().pb2_set_wait_budget_cycles(int(cycles)))


def wait_selftest(host_signal_sync: torch.Tensor, budget_cycles: int = 1 << 20) -> None:
    """Launch a kernel whose two warps wait on mbarriers that nothing
    completes, each with ``budget_cycles``: both waits run out, the error
    word of ``host_signal_sync`` becomes PB2_ERR_DEVICE_TIMEOUT and the
    kernel returns.  Asynchronous on the current stream."""
    if not host_signal_sync.is_cuda or host_signal_sync.numel() * host_signal_sync.element_size() < 16:
        _fail("host_signal_sync must be a CUDA buffer of at least 16 bytes")
    if not 0 < budget_cycles <= DEFAULT_WAIT_BUDGET_CYCLES:
        _fail(f"budget_cycles must be in (0, {DEFAULT_WAIT_BUDGET_CYCLES}]")
    L = _lib.load()
    with torch.cuda.device(host_signal_sync.device):
        st = L.pb2_wait_selftest(_device_index(host_signal_sync), int(budget_cycles),
                                 host_signal_sync.data_ptr(), _stream(host_signal_sync.device))
    _lib.check(st, "wait_selftest")
