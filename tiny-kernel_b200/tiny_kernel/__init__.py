"""tiny_kernel -- Python mirror of the reference's Zig kernel API over libtkcuda.

The reference (Lulzx/tiny-kernel) is used from Zig as::

    const device = try tk.init();                       // src/main.zig:17-19
    var x = try device.createBuffer(f32, K);            // src/metal/device.zig:85-87
    var q = try tk.kernels.quantized.QMatMulInt4.init(device);
    try q.forward(&x, &w, &s, &z, &out, m, k, n, group_size);   // quantized.zig:15-50

and this package reads the same way::

    import tiny_kernel as tk
    device = tk.init()
    x = device.create_buffer("f32", K)
    q = tk.kernels.quantized.QMatMulInt4.init(device)
    q.forward(x, w, s, z, out, m, k, n, group_size)

Buffers default to host-visible managed memory, like the reference's shared-storage
Metal buffers, so ``Buffer.slice()`` is a writable numpy view; ``forward`` is
synchronous, so results are visible on return.  Every kernel runs on the GPU through
``lib/libtkcuda.so``; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import TKError, check

_DTYPES = {
    "f32": np.float32,
    "f16": np.float16,
    "u8": np.uint8,
    "u16": np.uint16,
    "i32": np.int32,
    "u32": np.uint32,
}


class Buffer:
    """Typed device buffer, mirror of ``Buffer(T)`` (src/metal/device.zig:100-135)."""

    def __init__(self, device: "Device", dtype, count: int, kind: int = _lib.TK_MEM_SHARED):
        self.device = device
        self.dtype = np.dtype(_DTYPES.get(dtype, dtype))
        self.count = int(count)
        self.kind = kind
        self.nbytes = self.count * self.dtype.itemsize
        ptr = C.c_void_p()
        check(_lib.lib().tk_buffer_alloc(device.handle, max(self.nbytes, 16), kind,
                                         C.byref(ptr)))
        self.ptr = ptr.value

    @property
    def handle(self) -> int:
        return self.ptr

    def slice(self) -> np.ndarray:
        """Host view (managed/pinned buffers only), like Buffer.slice()."""
        if self.kind == _lib.TK_MEM_DEVICE:
            raise TKError(_lib.TK_ERR_ARG, "device-only buffer has no host view; use read()")
        self.device.synchronize()
        raw = (C.c_char * self.nbytes).from_address(self.ptr)
        return np.frombuffer(raw, dtype=self.dtype, count=self.count)

    constSlice = slice
    const_slice = slice

    def write(self, data) -> None:
        arr = np.ascontiguousarray(data, dtype=self.dtype).reshape(-1)
        if arr.size != self.count:
            raise ValueError(f"expected {self.count} elements, got {arr.size}")
        check(_lib.lib().tk_buffer_upload(self.device.handle, self.ptr,
                                          arr.ctypes.data_as(C.c_void_p), self.nbytes))

    def read(self) -> np.ndarray:
        out = np.empty(self.count, dtype=self.dtype)
        check(_lib.lib().tk_buffer_download(self.device.handle,
                                            out.ctypes.data_as(C.c_void_p), self.ptr,
                                            self.nbytes))
        return out

    def deinit(self) -> None:
        if self.ptr:
            check(_lib.lib().tk_buffer_free(self.device.handle, self.ptr))
            self.ptr = None

    def __del__(self):
        try:
            if self.ptr and self.device.handle:
                _lib.lib().tk_buffer_free(self.device.handle, self.ptr)
                self.ptr = None
        except Exception:
            pass


class Device:
    """Mirror of ``Device`` (src/metal/device.zig:4-98) over a CUDA device."""

    def __init__(self, ordinal: int = 0):
        h = C.c_void_p()
        check(_lib.lib().tk_device_create(int(ordinal), C.byref(h)))
        self.handle = h.value
        self.ordinal = ordinal

    def name(self) -> str:
        return _lib.lib().tk_device_name(self.handle).decode()

    def sm_count(self) -> int:
        return _lib.lib().tk_device_sm_count(self.handle)

    def launch_count(self) -> int:
        """Kernels enqueued through this device so far (graph captures included)."""
        return int(_lib.lib().tk_device_launch_count(self.handle))

    def stream(self) -> int:
        return _lib.lib().tk_device_stream(self.handle)

    def synchronize(self) -> None:
        check(_lib.lib().tk_device_synchronize(self.handle))

    def create_buffer(self, dtype, count: int, kind: int = _lib.TK_MEM_SHARED) -> Buffer:
        return Buffer(self, dtype, count, kind)

    createBuffer = create_buffer

    def create_buffer_with_data(self, dtype, data, kind: int = _lib.TK_MEM_SHARED) -> Buffer:
        arr = np.ascontiguousarray(data, dtype=_DTYPES.get(dtype, dtype)).reshape(-1)
        b = Buffer(self, arr.dtype, arr.size, kind)
        b.write(arr)
        return b

    createBufferWithData = create_buffer_with_data

    def deinit(self) -> None:
        if self.handle:
            _lib.lib().tk_device_destroy(self.handle)
            self.handle = None


def init(ordinal: int = 0) -> Device:
    """tk.init() (src/main.zig:17-19)."""
    return Device(ordinal)


def deinit(device: Device) -> None:
    """tk.deinit() (src/main.zig:21-23)."""
    device.deinit()


from . import kernels  # noqa: E402  (needs Device/Buffer above)

__all__ = ["init", "deinit", "Device", "Buffer", "TKError", "kernels"]
