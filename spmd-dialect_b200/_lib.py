"""ctypes binding of libspmdb200.so (the C ABI of include/spmd_b200.h).

The library is loaded from this package directory.  There is no fallback of
any kind: a missing or unloadable library raises at import time of the
binding, and every entry returning a non-zero status raises SpmdError.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
# SPMDB200_VARIANT=checked loads the checked build (run-time index checks that
# record instead of trapping; spmdb200_check_status reads the record).
VARIANT = os.environ.get("SPMDB200_VARIANT", "")
LIB_PATH = PKG_DIR / ("libspmdb200_checked.so" if VARIANT == "checked" else "libspmdb200.so")
CUBIN_PATH = PKG_DIR / "spmdb200_kernels.cubin"

c_p = ctypes.c_void_p
c_i = ctypes.c_int64
c_f = ctypes.c_float
c_sz = ctypes.c_size_t

# Unpacked memref descriptor argtypes (harness/run_host.py:41-65 convention).
D0 = [c_p, c_p, c_i]
D1 = [c_p, c_p, c_i, c_i, c_i]
D2 = [c_p, c_p, c_i, c_i, c_i, c_i, c_i]
D3 = [c_p, c_p, c_i, c_i, c_i, c_i, c_i, c_i, c_i]

STATUS = {
    0: "ok", -1: "invalid argument", -2: "CUDA error", -3: "device wait timed out",
    -4: "unsupported layout", -5: "bad workspace", -6: "no CUDA device", -7: "out-of-range access (checked build)",
}


class SpmdError(RuntimeError):
    """A libspmdb200 entry returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn}: {STATUS.get(status, status)} ({status}): {message}")
        self.status = status


# (name, restype, argtypes).  Device entries take a trailing cudaStream_t.
_SIGS = {
    # family A: reference-named host entries (void, like the SCF/OpenMP .so files)
    "ewise": (None, D1 + D1 + D1 + [c_i]),
    "stencil_cpu": (None, D2 + D2 + [c_i, c_i]),
    "atomic_sum": (None, D1 + D0 + [c_i]),
    "hierarchical_sum": (None, D1 + D0 + [c_i]),
    # family B: device entries
    "spmdb200_ewise": (ctypes.c_int, D1 + D1 + D1 + [c_i, c_p]),
    "spmdb200_axpy": (ctypes.c_int, [c_f] + D1 + D1 + [c_i, c_p]),
    "spmdb200_stencil3pt": (ctypes.c_int, D2 + D2 + [c_i, c_i, c_p]),
    "spmdb200_check_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint64)]),
    "spmdb200_forall_map": (ctypes.c_int, [ctypes.c_int, c_p, ctypes.c_int, c_p, c_p, c_p, c_p, c_p, ctypes.c_int,
                                           c_p, ctypes.c_int, ctypes.c_int, c_p]),
    "spmdb200_sum_workspace_bytes": (c_sz, [c_i]),
    "spmdb200_sum_f32": (ctypes.c_int, D1 + D0 + [c_i, c_p, c_sz, c_p]),
    "spmdb200_sum_f32_noalloc": (ctypes.c_int, D1 + D0 + [c_i, c_p]),
    "spmdb200_sum_i32": (ctypes.c_int, D1 + D0 + [c_i, c_p]),
    "spmdb200_hierarchical_sum": (ctypes.c_int, D1 + D0 + [c_i, c_p]),
    "spmdb200_reduction_status": (ctypes.c_int, []),
    "spmdb200_reduce_f32": (ctypes.c_int, [ctypes.c_int] + D1 + D0 + [c_i, c_f, c_p, c_sz, c_p]),
    "spmdb200_reduce_i32": (ctypes.c_int, [ctypes.c_int] + D1 + D0 + [c_i, ctypes.c_int32, c_p, c_sz, c_p]),
    "spmdb200_promotion_plan": (ctypes.c_int, [ctypes.c_int, c_p, c_p, c_p, c_p, c_i, c_i, ctypes.c_int, c_p, c_p]),
    "spmdb200_stencil_nd": (ctypes.c_int, [ctypes.c_int, c_p, c_p, c_p, c_p, c_p, c_p, ctypes.c_int, c_p, c_p, c_f,
                                           c_p, c_p, c_i, ctypes.c_int, c_p, c_p]),
    "spmdb200_sum_f32_partial": (ctypes.c_int, D1 + [c_i, c_p, c_p, c_sz, c_p]),
    "spmdb200_jacobi_workspace_bytes": (c_sz, []),
    "spmdb200_jacobi2d": (ctypes.c_int, D2 + D2 + [c_i, c_i, c_p, c_p, c_sz, c_p]),
    "spmdb200_jacobi3d": (ctypes.c_int, D3 + D3 + [c_i, c_i, c_p, c_p, c_sz, c_p]),
    "spmdb200_workspace_status": (ctypes.c_int, [c_p, c_p]),
    "spmdb200_set_wait_budget_ms": (ctypes.c_int, [c_i, c_i]),
    # multi-GPU row slabs
    "spmdb200_jacobi2d_slab": (ctypes.c_int, D2 + D2 + [c_i, c_i, c_i, c_i, c_p, c_p, c_p, c_p, c_p, c_i, c_p, c_p,
                                                       c_p, ctypes.c_int, ctypes.c_int, c_p, c_p, c_p]),
    "spmdb200_jacobi3d_slab": (ctypes.c_int, D3 + D3 + [c_i, c_i, c_i, c_i, c_p, c_p, c_p, c_p, c_p, c_i, c_p, c_p,
                                                       c_p, ctypes.c_int, ctypes.c_int, c_p, c_p, c_p]),
    "spmdb200_jacobi_slab_halo": (ctypes.c_int, [ctypes.c_int]),
    "spmdb200_jacobi_ws_reset": (ctypes.c_int, [c_p, c_p]),
    "spmdb200_jacobi2d_slab_residuals": (ctypes.c_int, [c_p, ctypes.c_int, c_i, c_p]),
    "spmdb200_dev_alloc": (ctypes.c_int, [c_sz, ctypes.POINTER(c_p)]),
    "spmdb200_dev_free": (ctypes.c_int, [c_p]),
    "spmdb200_memcpy": (ctypes.c_int, [c_p, c_p, c_sz, c_p]),
    "spmdb200_memcpy_async": (ctypes.c_int, [c_p, c_p, c_sz, c_p]),
    "spmdb200_ipc_handle": (ctypes.c_int, [c_p, c_p]),
    "spmdb200_ipc_open": (ctypes.c_int, [c_p, ctypes.POINTER(c_p)]),
    "spmdb200_ipc_close": (ctypes.c_int, [c_p]),
    "spmdb200_fill_jacobi_input": (ctypes.c_int, [c_p, c_i, c_i, c_i, c_i, c_i, ctypes.c_uint64, c_p]),
    "spmdb200_fill_jacobi3d_input": (ctypes.c_int, [c_p, c_i, c_i, c_i, c_i, c_i, c_i, c_i, ctypes.c_uint64, c_p]),
    # family C: end-to-end host entries
    "spmdb200_axpy_host": (ctypes.c_int, [c_f] + D1 + D1 + [c_i]),
    "spmdb200_sum_f32_host": (ctypes.c_int, D1 + D0 + [c_i]),
    "spmdb200_sum_i32_host": (ctypes.c_int, D1 + D0 + [c_i]),
    "spmdb200_jacobi2d_host": (ctypes.c_int, D2 + [c_i, c_i, c_p]),
    "spmdb200_jacobi2d_host_batch": (ctypes.c_int, [c_i, c_p, c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_p]),
    # utilities
    "spmdb200_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "spmdb200_last_error": (ctypes.c_int, []),
    "spmdb200_last_error_message": (ctypes.c_char_p, []),
    "spmdb200_version": (ctypes.c_char_p, []),
    "spmdb200_release_cache": (ctypes.c_int, []),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library with every signature set.  Raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python spmd-dialect_b200/build.py` "
                "(there is no CPU fallback for the B200 kernels)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(fn: str, status: int) -> None:
    if status != 0:
        msg = lib().spmdb200_last_error_message()
        raise SpmdError(fn, status, msg.decode() if msg else "")


def call(name: str, *args) -> int:
    """Calls a status-returning entry and raises SpmdError on failure."""
    st = getattr(lib(), name)(*args)
    check(name, st)
    return st
