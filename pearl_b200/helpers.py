"""Host-side helpers of the pearl_gemm package surface
(miner/pearl-gemm/src/pearl_gemm/helpers.py:14-82 and the pybind classes of
pearl_gemm_api.cpp:1021-1083): the pinned host-signal-header pool, the header
reader and the mapping of a hit to A rows / B columns."""

from __future__ import annotations

import ctypes
import enum
import logging
from collections import deque
from dataclasses import dataclass
from threading import Lock, Semaphore

import torch

from . import _lib
from .pearl_gemm_interface import make_pow_target_tensor  # noqa: F401  (re-export)

_LOG = logging.getLogger(__name__)


class HostSignalStatus(enum.IntEnum):
    kSignalIdle = 0
    kSignalTriggered = 1


class MMASize(ctypes.Structure):
    _fields_ = [("m", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int)]


class _HeaderLayout(ctypes.Structure):
    """Byte layout of HostSignalHeader (host_signal_header.hpp:21-50)."""

    _fields_ = [
        ("status", ctypes.c_int),
        ("gridDim", ctypes.c_uint32 * 3),
        ("blockDim", ctypes.c_uint32 * 3),
        ("blockIdx", ctypes.c_uint32 * 3),
        ("tileCoord", ctypes.c_uint32 * 3),
        ("threadIdx", ctypes.c_uint32 * 3),
        ("num_registers_per_thread", ctypes.c_uint16),
        ("thread_rows", ctypes.c_uint8 * 256),
        ("thread_cols", ctypes.c_uint8 * 256),
        ("mma_size", MMASize),
        ("mma_tile_size", MMASize),
        ("target", ctypes.c_uint32 * 8),
    ]


assert ctypes.sizeof(_HeaderLayout) <= _lib.HOST_SIGNAL_HEADER_SIZE


class HostSignalHeader:
    """Read-only view of a pinned host-signal header, with the attribute names
    of the reference's pybind class."""

    def __init__(self, raw: _HeaderLayout):
        self._raw = raw
        self.status = HostSignalStatus(raw.status) if raw.status in (0, 1) else raw.status
        self.gridDim = list(raw.gridDim)
        self.blockDim = list(raw.blockDim)
        self.blockIdx = list(raw.blockIdx)
        self.tileCoord = list(raw.tileCoord)
        self.threadIdx = list(raw.threadIdx)
        self.num_registers_per_thread = int(raw.num_registers_per_thread)
        self.mma_size = raw.mma_size
        self.mma_tile_size = raw.mma_tile_size
        self.target = list(raw.target)

    @property
    def thread_rows(self) -> memoryview:
        return memoryview(bytes(self._raw.thread_rows[: self.num_registers_per_thread]))

    @property
    def thread_cols(self) -> memoryview:
        return memoryview(bytes(self._raw.thread_cols[: self.num_registers_per_thread]))

    def __repr__(self) -> str:
        return (f"HostSignalHeader(status={int(self.status)}, tileCoord={self.tileCoord}, "
                f"mma_size=({self.mma_size.m}, {self.mma_size.n}, {self.mma_size.k}), "
                f"mma_tile_size=({self.mma_tile_size.m}, {self.mma_tile_size.n}, "
                f"{self.mma_tile_size.k}), num_registers_per_thread={self.num_registers_per_thread})")


def get_host_signal_header(host_signal_header_pinned: torch.Tensor) -> HostSignalHeader:
    """Copy of the header the kernel wrote (pearl_gemm_api.cpp:932-936)."""
    if host_signal_header_pinned.is_cuda:
        raise RuntimeError("host_signal_header_pinned must be a CPU (pinned) tensor")
    raw = _HeaderLayout.from_buffer_copy(
        host_signal_header_pinned.numpy().tobytes()[: ctypes.sizeof(_HeaderLayout)])
    return HostSignalHeader(raw)


def get_host_signal_header_size() -> int:
    return _lib.HOST_SIGNAL_HEADER_SIZE


def get_host_signal_sync_size() -> int:
    return _lib.HOST_SIGNAL_SYNC_SIZE


def get_host_signal_sync_fields(host_signal_sync: torch.Tensor) -> dict:
    """{lock, status, hit_count, error} of a host_signal_sync buffer (synchronizes)."""
    w = host_signal_sync.view(torch.int32).cpu().tolist()
    return {"lock": w[0], "status": w[1], "hit_count": w[2] & 0xFFFFFFFF, "error": w[3]}


class HostSignalHeaderPinnedPool:
    """Thread-safe pool of pinned header buffers (helpers.py:27-65)."""

    def __init__(self, pool_size: int = 128) -> None:
        self._pool_size = pool_size
        self._available_buffers = deque()
        self._used_buffers: set[int] = set()
        self._lock = Lock()
        self._semaphore = Semaphore(self._pool_size)
        size = get_host_signal_header_size()
        for _ in range(self._pool_size):
            self._available_buffers.append(torch.zeros((size,), dtype=torch.int8, pin_memory=True))

    def acquire(self) -> torch.Tensor:
        if not self._available_buffers:
            _LOG.warning("Pool size exceeded, self._pool_size=%d", self._pool_size)
        self._semaphore.acquire()
        with self._lock:
            buffer = self._available_buffers.popleft()
            if id(buffer) in self._used_buffers:
                raise AssertionError("Unexpectedly found available buffer in _used_buffers")
            self._used_buffers.add(id(buffer))
            return buffer

    def release(self, buffer: torch.Tensor) -> None:
        with self._lock:
            if id(buffer) not in self._used_buffers:
                raise ValueError("Attempted to release unused buffer")
            self._used_buffers.remove(id(buffer))
            self._available_buffers.append(buffer)
            buffer.zero_()
        self._semaphore.release()


@dataclass
class ProofTileIndices:
    A_row_indices: list[int]
    B_column_indices: list[int]


def extract_indices(header: HostSignalHeader) -> ProofTileIndices:
    """A rows and B columns of the hash tile a header reports (helpers.py:73-82)."""
    row0 = header.tileCoord[0] * header.mma_tile_size.m
    col0 = header.tileCoord[1] * header.mma_tile_size.n
    rows = sorted(set(header.thread_rows))
    cols = sorted(set(header.thread_cols))
    return ProofTileIndices(A_row_indices=[row0 + r for r in rows],
                            B_column_indices=[col0 + c for c in cols])
