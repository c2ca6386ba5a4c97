"""Device memory and host<->device copies over the C ABI.

`DeviceBuffer` owns one cudaMalloc allocation on one device; `PinnedBuffer` owns page-locked host
memory used as the staging area of the host<->device copies.  Both free their memory when closed
or garbage-collected.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


def set_device(device: int) -> None:
    _lib.call("mira_cuda_set_device", int(device))


def sync() -> None:
    _lib.call("mira_cuda_sync")


def device_info() -> tuple[int, int, int]:
    sm, ma, mi = C.c_int(), C.c_int(), C.c_int()
    _lib.call("mira_cuda_device_info", C.byref(sm), C.byref(ma), C.byref(mi))
    return sm.value, ma.value, mi.value


class DeviceBuffer:
    """`nbytes` of device memory on the device current at construction."""

    def __init__(self, nbytes: int, device: int | None = None, zero: bool = False):
        if device is not None:
            set_device(device)
        self.device = device
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        _lib.call("mira_cuda_malloc", C.byref(p), C.c_size_t(max(self.nbytes, 16)))
        self.ptr = int(p.value)
        if zero:
            _lib.call("mira_cuda_memset", C.c_void_p(self.ptr), 0, C.c_size_t(max(self.nbytes, 16)))

    @classmethod
    def from_array(cls, arr: np.ndarray, device: int | None = None) -> "DeviceBuffer":
        arr = np.ascontiguousarray(arr)
        buf = cls(arr.nbytes, device)
        buf.upload(arr)
        return buf

    def upload(self, arr: np.ndarray, offset: int = 0) -> None:
        arr = np.ascontiguousarray(arr)
        assert offset + arr.nbytes <= self.nbytes, "upload past the end of the buffer"
        _lib.call("mira_cuda_h2d", C.c_void_p(self.ptr + offset), C.c_void_p(arr.ctypes.data), C.c_size_t(arr.nbytes))
        # the copy is asynchronous: keep the source alive until the stream reaches it
        sync()

    def download(self, shape, dtype, offset: int = 0) -> np.ndarray:
        out = np.empty(shape, dtype)
        assert offset + out.nbytes <= self.nbytes, "download past the end of the buffer"
        _lib.call("mira_cuda_d2h", C.c_void_p(out.ctypes.data), C.c_void_p(self.ptr + offset), C.c_size_t(out.nbytes))
        sync()
        return out

    def close(self) -> None:
        if getattr(self, "ptr", 0):
            try:
                if self.device is not None:
                    set_device(self.device)
                _lib.call("mira_cuda_free", C.c_void_p(self.ptr))
            except Exception:
                pass
            self.ptr = 0

    def __del__(self):
        self.close()


class PinnedBuffer:
    """`nbytes` of page-locked host memory, viewable as a NumPy array."""

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        _lib.call("mira_cuda_host_alloc", C.byref(p), C.c_size_t(max(self.nbytes, 16)))
        self.ptr = int(p.value)

    def view(self, shape, dtype) -> np.ndarray:
        n = int(np.prod(shape, dtype=np.int64)) * np.dtype(dtype).itemsize
        assert n <= self.nbytes
        raw = (C.c_char * max(n, 1)).from_address(self.ptr)
        return np.frombuffer(raw, dtype=dtype, count=int(np.prod(shape, dtype=np.int64))).reshape(shape)

    def close(self) -> None:
        if getattr(self, "ptr", 0):
            try:
                _lib.call("mira_cuda_host_free", C.c_void_p(self.ptr))
            except Exception:
                pass
            self.ptr = 0

    def __del__(self):
        self.close()


class DeviceSlice:
    """The memory of `parent` from byte `offset` on (keeps the parent allocation alive)."""

    def __init__(self, parent, offset: int):
        self.parent = parent
        self.offset = int(offset)
        self.ptr = int(parent.ptr) + self.offset
        self.nbytes = parent.nbytes - self.offset


def ptr(x) -> C.c_void_p:
    """A C pointer from a DeviceBuffer, a DeviceSlice, an int address or None."""
    if x is None:
        return C.c_void_p(0)
    if isinstance(x, (DeviceBuffer, PinnedBuffer, DeviceSlice)):
        return C.c_void_p(x.ptr)
    return C.c_void_p(int(x))
