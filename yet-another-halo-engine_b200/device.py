"""Device memory, streams and events over the C ABI: the role of the reference's LoomDevice / LoomBuffer
(engine/model/loom_runtime.hpp:45-325), without PyTorch.

    dev = Device(0)
    buf = dev.upload(np_array)        # DeviceBuffer (owns device memory, freed on close / garbage collection)
    out = dev.empty(nbytes)
    host = buf.download(np.float32, shape)
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import check, lib


class DeviceBuffer:
    """A block of device memory owned by this object (freed by close() or on garbage collection)."""

    def __init__(self, dev: "Device", nbytes: int):
        self.dev = dev
        self.nbytes = int(nbytes)
        p = ctypes.c_void_p()
        check(lib().yah_malloc(ctypes.byref(p), max(self.nbytes, 1)))
        self.ptr = p.value

    def close(self):
        if self.ptr:
            lib().yah_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def upload(self, arr: np.ndarray, stream=None, offset: int = 0):
        a = np.ascontiguousarray(arr)
        if offset + a.nbytes > self.nbytes:
            raise ValueError("upload larger than the buffer")
        check(lib().yah_memcpy_h2d(self.ptr + offset, a.ctypes.data, a.nbytes, stream))
        if stream is None:
            self.dev.synchronize()
        return self

    def download(self, dtype, shape, stream=None, offset: int = 0) -> np.ndarray:
        out = np.empty(shape, dtype)
        if offset + out.nbytes > self.nbytes:
            raise ValueError("download larger than the buffer")
        check(lib().yah_memcpy_d2h(out.ctypes.data, self.ptr + offset, out.nbytes, stream))
        if stream is None:
            self.dev.synchronize()
        else:
            check(lib().yah_stream_synchronize(stream))
        return out

    def fill(self, byte: int, stream=None):
        check(lib().yah_memset(self.ptr, byte, self.nbytes, stream))
        return self


class PinnedBuffer:
    """Page-locked host memory viewed as a numpy array."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        check(lib().yah_host_alloc(ctypes.byref(p), max(int(nbytes), 1)))
        self.ptr = p.value
        self.nbytes = int(nbytes)

    def array(self, dtype, shape) -> np.ndarray:
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        if n > self.nbytes:
            raise ValueError("view larger than the pinned buffer")
        raw = (ctypes.c_uint8 * n).from_address(self.ptr)
        return np.frombuffer(raw, dtype=dtype, count=int(np.prod(shape))).reshape(shape)

    def close(self):
        if self.ptr:
            lib().yah_host_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Stream:
    def __init__(self):
        s = ctypes.c_void_p()
        check(lib().yah_stream_create(ctypes.byref(s)))
        self.handle = s.value

    def synchronize(self):
        check(lib().yah_stream_synchronize(self.handle))

    def wait(self, event: "Event"):
        """Later work on this stream waits for the work recorded on `event`."""
        check(lib().yah_stream_wait_event(self.handle, event.handle))

    def close(self):
        if self.handle:
            lib().yah_stream_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Event:
    def __init__(self):
        e = ctypes.c_void_p()
        check(lib().yah_event_create(ctypes.byref(e)))
        self.handle = e.value

    def record(self, stream=None):
        check(lib().yah_event_record(self.handle, stream))

    def synchronize(self):
        check(lib().yah_event_synchronize(self.handle))

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float()
        check(lib().yah_event_elapsed_ms(self.handle, end.handle, ctypes.byref(ms)))
        return float(ms.value)

    def close(self):
        if self.handle:
            lib().yah_event_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Graph:
    """A CUDA graph of the library calls made on `stream` between begin() and end(); launch() replays them."""

    def __init__(self, stream: "Stream"):
        self.stream = stream
        self.handle = None

    def begin(self):
        check(lib().yah_stream_begin_capture(self.stream.handle))

    def end(self):
        g = ctypes.c_void_p()
        check(lib().yah_stream_end_capture(self.stream.handle, ctypes.byref(g)))
        self.handle = g.value

    def launch(self):
        check(lib().yah_graph_launch(self.handle, self.stream.handle))

    def close(self):
        if self.handle:
            lib().yah_graph_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Device:
    """One CUDA device (made current on construction)."""

    def __init__(self, ordinal: int = 0):
        self.ordinal = ordinal
        check(lib().yah_set_device(ordinal))
        sm, ma, mi, mem = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        check(lib().yah_device_info(ordinal, ctypes.byref(sm), ctypes.byref(ma), ctypes.byref(mi), ctypes.byref(mem)))
        self.sm_count, self.cc, self.total_mem = sm.value, (ma.value, mi.value), mem.value

    def empty(self, nbytes: int) -> DeviceBuffer:
        return DeviceBuffer(self, nbytes)

    def upload(self, arr: np.ndarray, stream=None) -> DeviceBuffer:
        a = np.ascontiguousarray(arr)
        return DeviceBuffer(self, a.nbytes).upload(a, stream)

    def synchronize(self):
        check(lib().yah_device_synchronize())

    def status_word(self) -> int:
        """Read and clear the kernels' bounded-wait failure word (0 = no failure)."""
        c = ctypes.c_int()
        check(lib().yah_status_word(ctypes.byref(c)))
        return c.value


def device_count() -> int:
    n = ctypes.c_int()
    check(lib().yah_device_count(ctypes.byref(n)))
    return n.value
