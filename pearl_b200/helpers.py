"""Host-side helpers of the pearl_gemm package surface
(miner/pearl-gemm/src/pearl_gemm/helpers.py:14-82 and the pybind classes of
pearl_gemm_api.cpp:1021-1083): the pinned host-signal-header pool, the header
reader and the mapping of a hit to A rows / B columns."""

from __future__ import annotations

import ctypes
import enum
import logging
from dataclasses import dataclass
from threading import Lock

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
    """Pinned host-signal headers for concurrent mined GEMMs, with the
    reference pool's interface (helpers.py:27-65): ``acquire()`` hands out a
    zeroed 640-byte pinned int8 header and blocks while all ``pool_size``
    are out; ``release(buffer)`` zeroes it and returns it; both are safe to
    call from several threads.

    The headers are slots of ONE pinned allocation made up front (one
    page-locked region instead of ``pool_size`` small ones); the free slots
    wait in a blocking FIFO queue, and a released tensor is matched to its
    slot by its address, so a tensor that is not a slot of this pool, or a
    slot released twice, is refused with ValueError."""

    def __init__(self, pool_size: int = 128) -> None:
        import queue

        if pool_size <= 0:
            raise ValueError("pool_size must be positive")
        self._pool_size = pool_size
        size = get_host_signal_header_size()
        self._slab = torch.zeros((pool_size, size), dtype=torch.int8, pin_memory=True)
        self._slot_of = {int(self._slab[i].data_ptr()): i for i in range(pool_size)}
        self._out: set[int] = set()
        self._out_lock = Lock()
        self._free: "queue.Queue[int]" = queue.Queue()
        for i in range(pool_size):
            self._free.put(i)

    def acquire(self) -> torch.Tensor:
        if self._free.empty():
            _LOG.warning("all %d pinned headers are in use; waiting for a release", self._pool_size)
        slot = self._free.get()  # blocks until a header comes back
        with self._out_lock:
            self._out.add(slot)
        return self._slab[slot]

    def release(self, buffer: torch.Tensor) -> None:
        slot = self._slot_of.get(int(buffer.data_ptr())) if buffer.numel() == self._slab.shape[1] else None
        with self._out_lock:
            if slot is None or slot not in self._out:
                raise ValueError("release() got a header this pool has not handed out")
            self._out.discard(slot)
        self._slab[slot].zero_()
        self._free.put(slot)


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
