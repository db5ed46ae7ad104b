"""ctypes binding of oracle/_build/libspmd_oracle.so (built from spmd_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker the parity tests, the smoke check and
the CPU-baseline leg of the benchmark compare the B200 kernels against.  Every
function takes and returns numpy arrays and computes on the host.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import build as _build

c_p = ctypes.c_void_p
c_i = ctypes.c_int64
c_f = ctypes.c_float
D0 = [c_p, c_p, c_i]
D1 = [c_p, c_p, c_i, c_i, c_i]
D2 = [c_p, c_p, c_i, c_i, c_i, c_i, c_i]
D3 = [c_p, c_p, c_i, c_i, c_i, c_i, c_i, c_i, c_i]

_SIGS = {
    "ewise": (None, D1 + D1 + D1 + [c_i]),
    "stencil_cpu": (None, D2 + D2 + [c_i, c_i]),
    "atomic_sum": (None, D1 + D0 + [c_i]),
    "hierarchical_sum": (None, D1 + D0 + [c_i]),
    "hierarchical_sum_omp": (None, D1 + D0 + [c_i]),
    "oracle_axpy": (None, [c_f] + D1 + D1 + [c_i]),
    "oracle_sum_f64": (ctypes.c_double, D1 + [c_i]),
    "oracle_sum_i32": (ctypes.c_int32, D1 + [c_i]),
    "oracle_reduce_f32": (ctypes.c_float, [ctypes.c_int, c_p, c_i, c_f]),
    "oracle_reduce_i32": (ctypes.c_int32, [ctypes.c_int, c_p, c_i, ctypes.c_int32]),
    "oracle_jacobi2d_rows": (None, [c_p, c_p, c_i, c_i, c_i, c_i, c_i, c_i, c_p]),
    "oracle_jacobi2d": (None, D2 + D2 + [c_i, c_i, c_p]),
    "oracle_jacobi3d_planes": (None, [c_p, c_p, c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_p]),
    "oracle_jacobi3d_slab_planes": (None, [c_p, c_p, c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_p]),
    "oracle_jacobi3d": (None, D3 + D3 + [c_i, c_i, c_p]),
    "oracle_num_threads": (ctypes.c_int, []),
    "oracle_set_num_threads": (ctypes.c_int, [ctypes.c_int]),
    "oracle_forall_map": (None, [ctypes.c_int, c_p, ctypes.c_int, c_p, c_p, c_p, c_p, c_p, ctypes.c_int, c_p]),
    "oracle_stencil_nd": (None, [ctypes.c_int, c_p, c_p, c_p, c_p, c_p, c_p, ctypes.c_int, c_p, c_p, c_f, c_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        h = ctypes.CDLL(str(path))
        for n, (r, a) in _SIGS.items():
            f = getattr(h, n)
            f.restype, f.argtypes = r, a
        _lib = h
    return _lib


def lib_path() -> Path:
    return _build.OUT


def _p(a: np.ndarray) -> c_p:
    return a.ctypes.data_as(c_p)


def _d1(a: np.ndarray) -> tuple:
    es = a.itemsize
    return (_p(a), _p(a), c_i(0), c_i(a.shape[0]), c_i(a.strides[0] // es))


def _d2(a: np.ndarray) -> tuple:
    es = a.itemsize
    return (_p(a), _p(a), c_i(0), c_i(a.shape[0]), c_i(a.shape[1]), c_i(a.strides[0] // es), c_i(a.strides[1] // es))


def _d3(a: np.ndarray) -> tuple:
    es = a.itemsize
    return (_p(a), _p(a), c_i(0), *[c_i(s) for s in a.shape], *[c_i(s // es) for s in a.strides])


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> int:
    """OpenMP threads of later oracle calls on this thread (independent of
    OMP_NUM_THREADS); returns the count now in effect."""
    return int(lib().oracle_set_num_threads(int(n)))


def ewise(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    C = np.zeros(A.shape[0], dtype=np.float32)
    lib().ewise(*_d1(A), *_d1(B), *_d1(C), c_i(A.shape[0]))
    return C


def axpy(a: float, X: np.ndarray, Y: np.ndarray) -> np.ndarray:
    """Returns a new array a*X + Y (Y untouched)."""
    Z = np.array(Y, dtype=np.float32, copy=True)
    lib().oracle_axpy(c_f(a), *_d1(X), *_d1(Z), c_i(X.shape[0]))
    return Z


def stencil3(A: np.ndarray, N: int, M: int) -> np.ndarray:
    """B[i,j] = (A[i,j] + A[i,j+1]) + A[i+1,j] for i < N, j < M; reads off A are 0."""
    B = np.zeros((N, M), dtype=np.float32)
    lib().stencil_cpu(*_d2(A), *_d2(B), c_i(N), c_i(M))
    return B


def atomic_sum(A: np.ndarray, init: float = 0.0) -> np.float32:
    out = np.array([init], dtype=np.float32)
    lib().atomic_sum(*_d1(A), _p(out), _p(out), c_i(0), c_i(A.shape[0]))
    return out[0]


def hierarchical_sum(A: np.ndarray, init: float = 0.0) -> np.float32:
    out = np.array([init], dtype=np.float32)
    lib().hierarchical_sum(*_d1(A), _p(out), _p(out), c_i(0), c_i(A.shape[0]))
    return out[0]


def hierarchical_sum_omp(A: np.ndarray, init: float = 0.0) -> np.float32:
    """The OpenMP-lowering form (parallel tiles, atomic combine): timing baseline."""
    out = np.array([init], dtype=np.float32)
    lib().hierarchical_sum_omp(*_d1(A), _p(out), _p(out), c_i(0), c_i(A.shape[0]))
    return out[0]


def sum_f64(A: np.ndarray) -> float:
    return float(lib().oracle_sum_f64(*_d1(A), c_i(A.shape[0])))


def sum_i32(A: np.ndarray) -> int:
    return int(lib().oracle_sum_i32(*_d1(A), c_i(A.shape[0])))


KINDS = {"add": 0, "mul": 1, "max": 2, "min": 3, "and": 4, "or": 5, "xor": 6}


def reduce_f32(kind: str, A: np.ndarray, init: float) -> np.float32:
    A = np.ascontiguousarray(A, dtype=np.float32)
    return np.float32(lib().oracle_reduce_f32(KINDS[kind], _p(A), c_i(A.shape[0]), c_f(init)))


def reduce_i32(kind: str, A: np.ndarray, init: int) -> int:
    A = np.ascontiguousarray(A, dtype=np.int32)
    return int(lib().oracle_reduce_i32(KINDS[kind], _p(A), c_i(A.shape[0]), ctypes.c_int32(init)))


def jacobi2d(U0: np.ndarray, sweeps: int, res_every: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Returns (final grid, residuals) of `sweeps` sweeps from U0 (U0 untouched)."""
    U = np.array(U0, dtype=np.float32, copy=True, order="C")
    V = np.empty_like(U)
    nres = sweeps // res_every if res_every > 0 else 0
    res = np.zeros(max(nres, 1), dtype=np.float64)
    lib().oracle_jacobi2d(*_d2(U), *_d2(V), c_i(sweeps), c_i(res_every), _p(res))
    return (U if sweeps % 2 == 0 else V), res[:nres]


def jacobi2d_rows(u: np.ndarray, v: np.ndarray, row_lo: int, row_hi: int, g_row0: int, G: int,
                  want_res: bool = False) -> np.ndarray | None:
    """One sweep over local rows [row_lo, row_hi) of u into v (a row slab with halos)."""
    rr = np.zeros(max(row_hi - row_lo, 1), dtype=np.float64) if want_res else None
    lib().oracle_jacobi2d_rows(_p(u), _p(v), c_i(u.strides[0] // 4), c_i(u.shape[1]), c_i(row_lo), c_i(row_hi),
                               c_i(g_row0), c_i(G), _p(rr) if want_res else None)
    return rr


def jacobi3d(U0: np.ndarray, sweeps: int, res_every: int = 0) -> tuple[np.ndarray, np.ndarray]:
    U = np.array(U0, dtype=np.float32, copy=True, order="C")
    V = np.empty_like(U)
    nres = sweeps // res_every if res_every > 0 else 0
    res = np.zeros(max(nres, 1), dtype=np.float64)
    lib().oracle_jacobi3d(*_d3(U), *_d3(V), c_i(sweeps), c_i(res_every), _p(res))
    return (U if sweeps % 2 == 0 else V), res[:nres]


def jacobi3d_planes(u: np.ndarray, v: np.ndarray, z_lo: int, z_hi: int, g_z0: int, D: int,
                    want_res: bool = False) -> np.ndarray | None:
    """One sweep over local planes [z_lo, z_hi) of u into v (a z-slab of a D-plane
    grid whose local plane 0 is global plane g_z0; u, v C-contiguous)."""
    pr = np.zeros(max(z_hi - z_lo, 1), dtype=np.float64) if want_res else None
    lib().oracle_jacobi3d_slab_planes(_p(u), _p(v), c_i(g_z0), c_i(D), c_i(u.shape[1]), c_i(u.shape[2]),
                                      c_i(u.strides[0] // 4), c_i(u.strides[1] // 4), c_i(z_lo), c_i(z_hi),
                                      _p(pr) if want_res else None)
    return pr


def stencil_nd(A: np.ndarray, out_shape: tuple, offsets, weights=None, scale: float = 1.0, steps=None,
               out: np.ndarray | None = None) -> np.ndarray:
    """The general linear stencil on host arrays (see oracle_stencil_nd); B
    starts as `out` (or zeros) and only the step lattice is written."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    rank = A.ndim
    B = np.zeros(out_shape, np.float32) if out is None else np.array(out, np.float32, copy=True)
    off = np.ascontiguousarray(np.asarray(offsets, dtype=np.int64).reshape(-1, rank))
    i64 = lambda v: np.ascontiguousarray(np.asarray(v, dtype=np.int64))
    a_size, a_str = i64(A.shape), i64([s // 4 for s in A.strides])
    b_size, b_str = i64(B.shape), i64([s // 4 for s in B.strides])
    w = None if weights is None else np.ascontiguousarray(np.asarray(weights, np.float32))
    st = None if steps is None else i64(steps)
    lib().oracle_stencil_nd(rank, _p(A), _p(a_size), _p(a_str), _p(B), _p(b_size), _p(b_str), off.shape[0],
                            _p(off), _p(w) if w is not None else None, c_f(scale), _p(st) if st is not None else None)
    return B


def forall_map(inputs, out_shape, code, consts=(), out: np.ndarray | None = None) -> np.ndarray:
    """The general elementwise forall on host arrays (see oracle_forall_map):
    every point of out_shape gets the body program's STORE; inputs are arrays
    (any strides) of out_shape."""
    rank = len(out_shape)
    ins = [np.asarray(a, dtype=np.float32) for a in inputs]
    for a in ins:
        if a.shape != tuple(out_shape):
            raise ValueError("every input has the domain's shape")
    B = np.zeros(out_shape, np.float32) if out is None else out
    i64 = lambda v: np.ascontiguousarray(np.asarray(v, dtype=np.int64))
    ptrs = (c_p * max(len(ins), 1))(*[a.ctypes.data for a in ins])
    st = i64([s // 4 for a in ins for s in a.strides] or [0])
    words = np.ascontiguousarray(np.asarray([w for ins_ in code for w in ins_], dtype=np.int32))
    cs = np.ascontiguousarray(np.asarray(list(consts) or [0.0], dtype=np.float32))
    lib().oracle_forall_map(rank, _p(i64(out_shape)), len(ins), ctypes.cast(ptrs, c_p), _p(st), _p(B),
                            _p(i64([s // 4 for s in B.strides])), _p(words), len(code), _p(cs))
    return B
