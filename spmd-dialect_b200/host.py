"""Host-buffer (numpy) entry points, in the calling convention of the
reference's CPU harness (harness/run_host.py:30-75: unpacked descriptors built
from numpy arrays, ctypes CDLL, restype None).

The reference-named entries (`ewise`, `stencil_cpu`, `atomic_sum`,
`hierarchical_sum`) run on the current CUDA device: they copy the host
buffers in, launch the B200 kernel and copy the result back.  The void C
entries cannot return a status, so these wrappers read spmdb200_last_error()
and raise SpmdError -- the way harness/cuda_driver.py:43-59 raises
RuntimeError on any failed CUDA call.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import c_i, c_p, call, check, lib


def _ptr(arr: np.ndarray) -> c_p:
    return arr.ctypes.data_as(c_p)


def desc0d(arr: np.ndarray) -> tuple:
    p = _ptr(arr)
    return (p, p, c_i(0))


def desc1d(arr: np.ndarray, n: int | None = None) -> tuple:
    """(base, aligned, offset, size, stride) of a 1-D numpy array (any stride)."""
    if arr.ndim != 1:
        raise ValueError("rank-1 array expected")
    es = arr.itemsize
    if arr.strides[0] % es or arr.strides[0] <= 0:
        raise ValueError("positive element-multiple stride expected")
    p = _ptr(arr)
    return (p, p, c_i(0), c_i(arr.shape[0] if n is None else n), c_i(arr.strides[0] // es))


def desc2d(arr: np.ndarray) -> tuple:
    """(base, aligned, offset, size0, size1, stride0, stride1) of a 2-D numpy array."""
    if arr.ndim != 2:
        raise ValueError("rank-2 array expected")
    es = arr.itemsize
    s0, s1 = arr.strides
    if s0 % es or s1 % es or s0 <= 0 or s1 <= 0:
        raise ValueError("positive element-multiple strides expected")
    p = _ptr(arr)
    return (p, p, c_i(0), c_i(arr.shape[0]), c_i(arr.shape[1]), c_i(s0 // es), c_i(s1 // es))


def _void(name: str, *args) -> None:
    getattr(lib(), name)(*args)
    check(name, lib().spmdb200_last_error())


# ---- reference-named entries (GPU compute, host buffers) -------------------------
def ewise(A: np.ndarray, B: np.ndarray, C: np.ndarray, N: int | None = None) -> np.ndarray:
    N = A.shape[0] if N is None else N
    _void("ewise", *desc1d(A), *desc1d(B), *desc1d(C), c_i(N))
    return C


def stencil_cpu(A: np.ndarray, B: np.ndarray, N: int | None = None, M: int | None = None) -> np.ndarray:
    N = B.shape[0] if N is None else N
    M = B.shape[1] if M is None else M
    _void("stencil_cpu", *desc2d(A), *desc2d(B), c_i(N), c_i(M))
    return B


def atomic_sum(A: np.ndarray, out: np.ndarray, N: int | None = None) -> np.ndarray:
    _void("atomic_sum", *desc1d(A), *desc0d(out), c_i(A.shape[0] if N is None else N))
    return out


def hierarchical_sum(A: np.ndarray, out: np.ndarray, N: int | None = None) -> np.ndarray:
    _void("hierarchical_sum", *desc1d(A), *desc0d(out), c_i(A.shape[0] if N is None else N))
    return out


# ---- end-to-end entries for the configurations without a reference entry --------
def axpy_host(alpha: float, x: np.ndarray, y: np.ndarray) -> np.ndarray:
    call("spmdb200_axpy_host", ctypes.c_float(alpha), *desc1d(x), *desc1d(y), c_i(x.shape[0]))
    return y


def sum_f32_host(A: np.ndarray, out: np.ndarray) -> np.ndarray:
    call("spmdb200_sum_f32_host", *desc1d(A), *desc0d(out), c_i(A.shape[0]))
    return out


def sum_i32_host(A: np.ndarray, out: np.ndarray) -> np.ndarray:
    call("spmdb200_sum_i32_host", *desc1d(A), *desc0d(out), c_i(A.shape[0]))
    return out


def jacobi2d_host(U: np.ndarray, sweeps: int, res_every: int = 0) -> tuple[np.ndarray, np.ndarray | None]:
    """Runs `sweeps` sweeps on U in place (host buffer); returns (U, residuals)."""
    nres = sweeps // res_every if res_every > 0 else 0
    res = np.zeros(max(nres, 1), dtype=np.float64)
    call("spmdb200_jacobi2d_host", *desc2d(U), c_i(sweeps), c_i(res_every), _ptr(res))
    return U, (res[:nres] if nres else None)


def jacobi2d_host_batch(grids: list[np.ndarray], sweeps: int, res_every: int = 0) -> list:
    """Runs `sweeps` sweeps on each host grid in place, the copies of one grid
    overlapping the sweeps of its neighbours in the list (pinned grids, e.g.
    torch.empty(..., pin_memory=True).numpy(), overlap; pageable ones do not).
    Every grid has the same shape and row pitch.  Returns one residual array
    (or None) per grid."""
    if not grids:
        return []
    g0 = grids[0]
    if g0.ndim != 2 or g0.dtype != np.float32 or g0.strides[1] != 4 or g0.strides[0] % 4:
        raise ValueError("float32 grids with contiguous rows expected")
    for g in grids:
        if g.shape != g0.shape or g.strides != g0.strides or g.dtype != g0.dtype:
            raise ValueError("every grid of a batch must share shape, strides and dtype")
    nres = sweeps // res_every if res_every > 0 else 0
    res = [np.zeros(max(nres, 1), dtype=np.float64) for _ in grids]
    ptrs = (c_p * len(grids))(*[g.ctypes.data for g in grids])
    rptr = (c_p * len(grids))(*[r.ctypes.data for r in res])
    call("spmdb200_jacobi2d_host_batch", c_i(len(grids)), ctypes.cast(ptrs, c_p), c_i(0), c_i(g0.shape[0]),
         c_i(g0.shape[1]), c_i(g0.strides[0] // 4), c_i(1), c_i(sweeps), c_i(res_every), ctypes.cast(rptr, c_p))
    return [r[:nres] if nres else None for r in res]
