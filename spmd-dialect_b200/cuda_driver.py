"""Minimal CUDA driver-API client with the public surface of the reference's
harness/cuda_driver.py (init / load_ptx / get_function / alloc / memcpy_h2d /
memcpy_d2h / memset / launch / synchronize / event_*), so code written against
that harness runs unchanged against spmdb200_kernels.cubin.

Differences from the reference module, by design:
  * init() retains the device's PRIMARY context instead of creating a new one,
    so buffers and streams interoperate with the CUDA runtime (torch and
    libspmdb200.so use the primary context too);
  * load_ptx() accepts any image cuModuleLoadData takes (PTX text or a cubin);
    load_cubin() is the same call under a clearer name.
Kernel arguments: DevicePtr -> u64, Python int / numpy integer -> i64,
Python float / numpy float32 -> f32 (the reference's marshalling rule).
"""
from __future__ import annotations

import ctypes
import ctypes.util

import numpy as np

_cuda = None


def _driver() -> ctypes.CDLL:
    global _cuda
    if _cuda is None:
        name = ctypes.util.find_library("cuda") or "libcuda.so.1"
        _cuda = ctypes.CDLL(name)
    return _cuda


def _check(res: int, what: str) -> None:
    if res != 0:
        cu = _driver()
        nm, ds = ctypes.c_char_p(), ctypes.c_char_p()
        cu.cuGetErrorName(res, ctypes.byref(nm))
        cu.cuGetErrorString(res, ctypes.byref(ds))
        raise RuntimeError(f"CUDA driver error {res} in {what}: "
                           f"{(nm.value or b'?').decode()} - {(ds.value or b'?').decode()}")


def _call(fn: str, *args) -> None:
    f = getattr(_driver(), fn)
    _check(f(*args), fn)


class DevicePtr:
    """A CUdeviceptr plus its size in bytes."""

    def __init__(self, addr: int, nbytes: int):
        self._addr = ctypes.c_uint64(addr)
        self.nbytes = nbytes

    @property
    def addr(self) -> ctypes.c_uint64:
        return self._addr

    @property
    def addr_int(self) -> int:
        return self._addr.value

    def free(self) -> None:
        if self._addr.value:
            _call("cuMemFree_v2", self._addr)
            self._addr = ctypes.c_uint64(0)

    def __repr__(self) -> str:
        return f"DevicePtr(0x{self._addr.value:x}, {self.nbytes}B)"


_ctx = None


def init(device: int = 0) -> None:
    """Initialises the driver and makes the device's primary context current."""
    global _ctx
    if _ctx is not None:
        return
    _call("cuInit", ctypes.c_uint(0))
    dev = ctypes.c_int(0)
    _call("cuDeviceGet", ctypes.byref(dev), ctypes.c_int(device))
    ctx = ctypes.c_void_p()
    _call("cuDevicePrimaryCtxRetain", ctypes.byref(ctx), dev)
    _call("cuCtxSetCurrent", ctx)
    _ctx = ctx


def load_ptx(path: str):
    """cuModuleLoadData on the file's bytes (PTX or cubin); returns the CUmodule."""
    with open(path, "rb") as fh:
        image = fh.read()
    if not image.endswith(b"\0") and image[:4] != b"\x7fELF":
        image += b"\0"  # PTX text must be NUL-terminated
    buf = ctypes.create_string_buffer(image, len(image))
    mod = ctypes.c_void_p()
    _call("cuModuleLoadData", ctypes.byref(mod), buf)
    return mod


load_cubin = load_ptx


def get_function(module, name: str):
    fn = ctypes.c_void_p()
    _call("cuModuleGetFunction", ctypes.byref(fn), module, name.encode())
    return fn


def alloc(n_bytes: int) -> DevicePtr:
    p = ctypes.c_uint64(0)
    _call("cuMemAlloc_v2", ctypes.byref(p), ctypes.c_size_t(max(int(n_bytes), 1)))
    return DevicePtr(p.value, int(n_bytes))


def memcpy_h2d(dst: DevicePtr, src: np.ndarray) -> None:
    a = np.ascontiguousarray(src)
    _call("cuMemcpyHtoD_v2", dst.addr, a.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(a.nbytes))


def memcpy_d2h(dst: np.ndarray, src: DevicePtr) -> None:
    if not dst.flags["C_CONTIGUOUS"]:
        raise ValueError("destination must be C-contiguous")
    if dst.nbytes != src.nbytes:
        raise ValueError(f"size mismatch: dst={dst.nbytes}, src={src.nbytes}")
    _call("cuMemcpyDtoH_v2", dst.ctypes.data_as(ctypes.c_void_p), src.addr, ctypes.c_size_t(dst.nbytes))


def memset(dst: DevicePtr, value: int, n_bytes: int) -> None:
    _call("cuMemsetD8_v2", dst.addr, ctypes.c_ubyte(value), ctypes.c_size_t(n_bytes))


def _marshal(a):
    if isinstance(a, DevicePtr):
        return ctypes.c_uint64(a.addr_int)
    if isinstance(a, (bool, np.bool_)):
        raise TypeError("bool kernel arguments are not supported")
    if isinstance(a, (int, np.integer)):
        return ctypes.c_int64(int(a))
    if isinstance(a, (float, np.floating)):
        return ctypes.c_float(float(a))
    raise TypeError(f"unsupported kernel argument type {type(a)}")


def launch(fn, grid, block, *args, shared_bytes: int = 0, stream=None) -> None:
    vals = [_marshal(a) for a in args]
    params = (ctypes.c_void_p * max(len(vals), 1))(*[ctypes.cast(ctypes.byref(v), ctypes.c_void_p) for v in vals])
    g = tuple(grid) + (1,) * (3 - len(grid))
    b = tuple(block) + (1,) * (3 - len(block))
    _call("cuLaunchKernel", fn, ctypes.c_uint(g[0]), ctypes.c_uint(g[1]), ctypes.c_uint(g[2]),
          ctypes.c_uint(b[0]), ctypes.c_uint(b[1]), ctypes.c_uint(b[2]), ctypes.c_uint(shared_bytes),
          ctypes.c_void_p(stream), params, ctypes.c_void_p(0))


def synchronize() -> None:
    _call("cuCtxSynchronize")


def event_create():
    ev = ctypes.c_void_p()
    _call("cuEventCreate", ctypes.byref(ev), ctypes.c_uint(0))
    return ev


def event_record(event, stream=None) -> None:
    _call("cuEventRecord", event, ctypes.c_void_p(stream))


def event_elapsed_ms(start, stop) -> float:
    _call("cuEventSynchronize", stop)
    ms = ctypes.c_float(0.0)
    _call("cuEventElapsedTime", ctypes.byref(ms), start, stop)
    return float(ms.value)


def event_destroy(event) -> None:
    _call("cuEventDestroy_v2", event)
