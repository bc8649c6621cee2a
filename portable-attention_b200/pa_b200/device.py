"""Device memory, streams, events and page-locked host arrays over the C ABI.

Everything here is plumbing around ``pa_malloc`` / ``pa_memcpy_*`` /
``pa_stream_*`` / ``pa_event_*`` (include/pa_b200.h). No PyTorch: the backend
keeps the reference project's ctypes-only runtime footprint.
"""

from __future__ import annotations

import ctypes
import threading
import weakref

import numpy as np

from ._lib import check, lib

__all__ = [
    "DeviceArena", "DeviceBuffer", "Event", "PinnedPool", "Stream", "current_device",
    "device_count", "is_pinned", "pinned_empty", "set_device", "sync_device_status",
]

_ALIGN = 256


def device_count() -> int:
    """Visible CUDA devices (0 when there is no usable GPU or driver)."""
    n = ctypes.c_int32(0)
    status = lib().pa_init(ctypes.byref(n))
    return int(n.value) if status == 0 else 0


def set_device(dev: int) -> None:
    check(lib().pa_set_device(int(dev)))


def current_device() -> int:
    d = ctypes.c_int32(0)
    check(lib().pa_get_device(ctypes.byref(d)))
    return int(d.value)


def sync_device_status() -> None:
    """Raise if a bounded device-side wait gave up since the last check."""
    code = ctypes.c_int32(0)
    check(lib().pa_device_status(ctypes.byref(code)))


class Stream:
    """A non-blocking CUDA stream owned by the library."""

    def __init__(self) -> None:
        h = ctypes.c_void_p()
        check(lib().pa_stream_create(ctypes.byref(h)))
        self.handle = h.value
        self._fin = weakref.finalize(self, lib().pa_stream_destroy, h.value)

    def synchronize(self) -> None:
        check(lib().pa_stream_sync(self.handle))

    def close(self) -> None:
        self._fin()


class Event:
    """A CUDA event for device-side timing."""

    def __init__(self) -> None:
        h = ctypes.c_void_p()
        check(lib().pa_event_create(ctypes.byref(h)))
        self.handle = h.value
        self._fin = weakref.finalize(self, lib().pa_event_destroy, h.value)

    def synchronize(self) -> None:
        check(lib().pa_event_sync(self.handle))

    def record(self, stream: Stream | None = None) -> None:
        check(lib().pa_event_record(self.handle, stream.handle if stream else None))

    def wait_on(self, stream: Stream) -> None:
        """Make later work on ``stream`` wait until this event has completed."""
        check(lib().pa_stream_wait_event(stream.handle, self.handle))

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0.0)
        check(lib().pa_event_elapsed_ms(self.handle, end.handle, ctypes.byref(ms)))
        return float(ms.value)


class DeviceBuffer:
    """One device allocation; freed when garbage-collected or on :meth:`free`."""

    def __init__(self, nbytes: int) -> None:
        p = ctypes.c_void_p()
        check(lib().pa_malloc(ctypes.byref(p), max(int(nbytes), 1)))
        self.ptr = p.value
        self.nbytes = int(nbytes)
        self._fin = weakref.finalize(self, lib().pa_free, p.value)

    def free(self) -> None:
        self._fin()
        self.ptr = None


class DeviceArena:
    """A grow-only device allocation carved into 256-byte aligned pieces per call.

    The numpy-facing backend is synchronous, so one arena per device serves
    every call in turn (guarded by a lock) and saves a cudaMalloc per call.
    """

    def __init__(self) -> None:
        self._buf: DeviceBuffer | None = None
        self.lock = threading.Lock()

    def carve(self, sizes: list[int]) -> list[int]:
        offs, total = [], 0
        for s in sizes:
            offs.append(total)
            total += (int(s) + _ALIGN - 1) // _ALIGN * _ALIGN
        if self._buf is None or self._buf.nbytes < total:
            if self._buf is not None:
                self._buf.free()
            self._buf = DeviceBuffer(max(total, 1 << 20))
        return [self._buf.ptr + o for o in offs]

    def release(self) -> None:
        if self._buf is not None:
            self._buf.free()
            self._buf = None


class _PinnedBlock:
    """One page-locked host allocation (freed when dropped by its pool)."""

    def __init__(self, nbytes: int) -> None:
        p = ctypes.c_void_p()
        check(lib().pa_host_alloc(ctypes.byref(p), max(int(nbytes), 1)))
        self.ptr = p.value
        self.nbytes = int(nbytes)
        self._fin = weakref.finalize(self, lib().pa_host_free, p.value)


class PinnedPool:
    """Reuses page-locked host blocks: pinning is slow, so arrays handed out by
    :meth:`array` give their block back to the pool (not to the OS) once the
    array and every view of it are gone. At most ``cap`` bytes stay cached."""

    GRANULE = 2 << 20

    def __init__(self, cap: int = 8 << 30) -> None:
        self._free: dict[int, list[_PinnedBlock]] = {}
        self._cached = 0
        self._cap = cap
        self._lock = threading.Lock()

    def array(self, shape, dtype) -> np.ndarray:
        dt = np.dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        size = max(self.GRANULE, (n + self.GRANULE - 1) // self.GRANULE * self.GRANULE)
        with self._lock:
            bucket = self._free.get(size)
            block = bucket.pop() if bucket else None
            if block is not None:
                self._cached -= size
        if block is None:
            block = _PinnedBlock(size)
        raw = (ctypes.c_byte * max(n, 1)).from_address(block.ptr)
        weakref.finalize(raw, self._give_back, block)
        return np.frombuffer(raw, dtype=np.uint8, count=n).view(dt).reshape(shape)

    def _give_back(self, block: _PinnedBlock) -> None:
        with self._lock:
            if self._cached + block.nbytes <= self._cap:
                self._free.setdefault(block.nbytes, []).append(block)
                self._cached += block.nbytes
                return
        block._fin()


_pool = PinnedPool()


def is_pinned(arr: np.ndarray) -> bool:
    """True when the array's memory is page-locked (fast, asynchronous copies)."""
    flag = ctypes.c_int32(0)
    check(lib().pa_host_is_pinned(arr.ctypes.data, ctypes.byref(flag)))
    return bool(flag.value)


def pinned_empty(shape, dtype) -> np.ndarray:
    """An uninitialised NumPy array in page-locked host memory (fast H2D/D2H).

    The block returns to a process-wide pool when the array (and every view
    of it) is gone, so repeated calls of the same size do not re-pin memory.
    """
    return _pool.array(shape, dtype)
