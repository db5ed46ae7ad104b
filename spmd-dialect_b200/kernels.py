"""Device-memory entry points over torch tensors (PyTorch = allocator + streams).

Each function builds the unpacked memref descriptors the C ABI expects from a
CUDA tensor (aligned pointer = tensor.data_ptr(), offset 0, sizes and strides
in elements) and calls the matching spmdb200_* entry on the current stream.
All compute happens in libspmdb200.so; nothing here computes anything.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import c_i, c_p, call, lib
from .forall_program import insn as map_insn  # noqa: F401  (re-exported)

_DTYPES = {torch.float32: "f32", torch.int32: "i32", torch.uint8: "u8", torch.float64: "f64"}


def memref(t: torch.Tensor) -> tuple:
    """Unpacked memref descriptor (base, aligned, offset, sizes..., strides...)."""
    if not t.is_cuda:
        raise ValueError("device entries take CUDA tensors")
    if t.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {t.dtype}")
    p = c_p(t.data_ptr())
    return (p, p, c_i(0), *[c_i(s) for s in t.shape], *[c_i(s) for s in t.stride()])


def _stream(stream) -> c_p:
    s = torch.cuda.current_stream() if stream is None else stream
    return c_p(s.cuda_stream)


def ewise(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """out = a + b (f32), the ewise_kernel forall."""
    n = a.shape[0]
    out = torch.empty_like(a) if out is None else out
    call("spmdb200_ewise", *memref(a), *memref(b), *memref(out), c_i(n), _stream(stream))
    return out


def axpy(alpha: float, x: torch.Tensor, y: torch.Tensor, stream=None) -> torch.Tensor:
    """y = fadd(fmul(alpha, x), y) in place."""
    call("spmdb200_axpy", ctypes.c_float(alpha), *memref(x), *memref(y), c_i(x.shape[0]), _stream(stream))
    return y


def stencil3pt(a: torch.Tensor, out: torch.Tensor, n: int | None = None, m: int | None = None,
               stream=None) -> torch.Tensor:
    """out[i,j] = (a[i,j] + a[i,j+1]) + a[i+1,j] for i < n, j < m (reads off `a` are 0)."""
    n = out.shape[0] if n is None else n
    m = out.shape[1] if m is None else m
    call("spmdb200_stencil3pt", *memref(a), *memref(out), c_i(n), c_i(m), _stream(stream))
    return out


PLAN_REASONS = {0: "promote", 1: "unbounded offsets", 2: "read-write operand", 3: "footprint too large",
                4: "no reuse"}


def _i64(vals) -> ctypes.Array:
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * max(len(vals), 1))(*vals)


def promotion_plan(tile_sizes, min_offsets, max_offsets, steps=None, elem_bytes: int = 4,
                   max_group_bytes: int = 49152, read_only: bool = True) -> tuple[int, tuple, int]:
    """(plan code, footprint extents, footprint bytes) of one operand, as the
    reference's computePromotionPlan decides it (host only, no GPU needed)."""
    rank = len(tile_sizes)
    dims = (ctypes.c_int64 * 3)()
    nbytes = ctypes.c_int64(0)
    code = lib().spmdb200_promotion_plan(rank, _i64(tile_sizes), _i64(steps) if steps is not None else None,
                                         _i64(min_offsets), _i64(max_offsets), c_i(elem_bytes),
                                         c_i(max_group_bytes), int(bool(read_only)), dims, ctypes.byref(nbytes))
    if code < 0:
        from ._lib import check
        check("spmdb200_promotion_plan", code)  # raises with the library's message
    return int(code), tuple(int(dims[d]) for d in range(rank)), int(nbytes.value)


def stencil_nd(a: torch.Tensor, out: torch.Tensor, offsets, weights=None, scale: float = 1.0, tile_sizes=None,
               steps=None, max_group_bytes: int = 0, policy: int = 0, stream=None) -> bool:
    """out[p] = scale * sum_k w_k * a[p + offsets[k]] in order, for p on the step
    lattice inside out's shape (reads off `a` are 0).  Returns True when the
    promotion plan staged tiles in shared memory."""
    rank = a.dim()
    if out.dim() != rank or not (1 <= rank <= 3):
        raise ValueError("a and out must have the same rank, 1-3")
    offs = [int(v) for row in offsets for v in (row if hasattr(row, "__len__") else [row])]
    ntaps = len(offs) // rank
    tile_sizes = tile_sizes or ([256] if rank == 1 else [32, 8] if rank == 2 else [8, 8, 4])
    w = None if weights is None else (ctypes.c_float * ntaps)(*[float(x) for x in weights])
    promoted = ctypes.c_int(0)
    call("spmdb200_stencil_nd", rank, c_p(a.data_ptr()), _i64(a.shape), _i64(a.stride()), c_p(out.data_ptr()),
         _i64(out.shape), _i64(out.stride()), ntaps, _i64(offs), w, ctypes.c_float(scale), _i64(tile_sizes),
         _i64(steps) if steps is not None else None, c_i(max_group_bytes), policy, ctypes.byref(promoted),
         _stream(stream))
    return bool(promoted.value)


def forall_map(inputs, out: torch.Tensor, code, consts=(), n_regs: int | None = None, stream=None) -> torch.Tensor:
    """out[p] = f(inputs[0][p], ...) over out's domain (rank 1-3), f the
    straight-line program `code` (a list of forall_program.insn pairs; LOADs
    first, one STORE last).  Each input is a view with out's shape."""
    rank = out.dim()
    if not 1 <= rank <= 3:
        raise ValueError("forall_map: rank 1-3")
    for t in inputs:
        if tuple(t.shape) != tuple(out.shape) or t.dtype != torch.float32 or not t.is_cuda:
            raise ValueError("forall_map: every input is a CUDA f32 view with out's shape")
    if out.dtype != torch.float32 or not out.is_cuda:
        raise ValueError("forall_map: out must be a CUDA f32 tensor")
    words = [int(w) for ins in code for w in ins]
    if n_regs is None:
        n_regs = 1 + max(max((w0 >> 8) & 255, (w0 >> 16) & 255, (w0 >> 24) & 255) for w0 in words[0::2])
    ptrs = (c_p * max(len(inputs), 1))(*[t.data_ptr() for t in inputs])
    strides = _i64([s for t in inputs for s in t.stride()] or [0])
    cs = (ctypes.c_float * max(len(consts), 1))(*[float(c) for c in consts])
    call("spmdb200_forall_map", rank, _i64(out.shape), len(inputs), ptrs, strides, c_p(out.data_ptr()),
         _i64(out.stride()), (ctypes.c_int32 * len(words))(*words), len(code), cs, len(consts), n_regs,
         _stream(stream))
    return out


def sum_workspace(n: int, device=None) -> torch.Tensor:
    """Zero-filled workspace for sum_f32 (reusable: every call leaves it zeroed)."""
    nbytes = int(lib().spmdb200_sum_workspace_bytes(c_i(n)))
    return torch.zeros(nbytes, dtype=torch.uint8, device=device or "cuda")


def sum_f32(a: torch.Tensor, out: torch.Tensor, ws: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """out[0] = f32(f64(out[0]) + sum(a)), deterministic."""
    n = a.shape[0]
    ws = sum_workspace(n, a.device) if ws is None else ws
    o = c_p(out.data_ptr())
    call("spmdb200_sum_f32", *memref(a), o, o, c_i(0), c_i(n), c_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
         _stream(stream))
    return out


def sum_i32(a: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
    """out[0] += sum(a) in wrapping int32."""
    o = c_p(out.data_ptr())
    call("spmdb200_sum_i32", *memref(a), o, o, c_i(0), c_i(a.shape[0]), _stream(stream))
    return out


def hierarchical_sum(a: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
    """out[0] += sum(a) with one f32 atomic per block (reference semantics)."""
    o = c_p(out.data_ptr())
    call("spmdb200_hierarchical_sum", *memref(a), o, o, c_i(0), c_i(a.shape[0]), _stream(stream))
    return out


KINDS = {"add": 0, "mul": 1, "max": 2, "min": 3, "and": 4, "or": 5, "xor": 6}


def reduce(kind: str, a: torch.Tensor, init, out: torch.Tensor | None = None, ws: torch.Tensor | None = None,
           stream=None) -> torch.Tensor:
    """out[0] = init (+) a[0] (+) ... for an spmd.reduce kind (f32: add/mul/max/min; i32: all seven)."""
    n = a.shape[0]
    out = torch.empty(1, dtype=a.dtype, device=a.device) if out is None else out
    ws = sum_workspace(n, a.device) if ws is None else ws
    o = c_p(out.data_ptr())
    common = (*memref(a), o, o, c_i(0), c_i(n))
    if a.dtype == torch.float32:
        call("spmdb200_reduce_f32", ctypes.c_int(KINDS[kind]), *common, ctypes.c_float(init), c_p(ws.data_ptr()),
             ctypes.c_size_t(ws.numel()), _stream(stream))
    elif a.dtype == torch.int32:
        call("spmdb200_reduce_i32", ctypes.c_int(KINDS[kind]), *common, ctypes.c_int32(init), c_p(ws.data_ptr()),
             ctypes.c_size_t(ws.numel()), _stream(stream))
    else:
        raise TypeError("reduce takes float32 or int32 tensors")
    return out


def jacobi_workspace(device=None) -> torch.Tensor:
    return torch.zeros(int(lib().spmdb200_jacobi_workspace_bytes()), dtype=torch.uint8, device=device or "cuda")


def workspace_status(ws: torch.Tensor, stream=None) -> None:
    """Synchronises and raises SpmdError if the run left a device-side timeout."""
    call("spmdb200_workspace_status", c_p(ws.data_ptr()), _stream(stream))


def _jacobi(entry: str, u: torch.Tensor, v: torch.Tensor, sweeps: int, res_every: int,
            ws: torch.Tensor | None, res: torch.Tensor | None, check: bool, stream):
    ws = jacobi_workspace(u.device) if ws is None else ws
    nres = sweeps // res_every if res_every > 0 else 0
    if res is None and nres > 0:
        res = torch.zeros(nres, dtype=torch.float64, device=u.device)
    rp = c_p(res.data_ptr()) if res is not None else c_p(0)
    call(entry, *memref(u), *memref(v), c_i(sweeps), c_i(res_every), rp, c_p(ws.data_ptr()),
         ctypes.c_size_t(ws.numel()), _stream(stream))
    if check:
        workspace_status(ws, stream)
    return (u if sweeps % 2 == 0 else v), res


def jacobi2d(u: torch.Tensor, v: torch.Tensor, sweeps: int, res_every: int = 0, ws=None, res=None,
             check: bool = True, stream=None):
    """`sweeps` 5-point sweeps ping-ponging u -> v -> u ...; returns (final grid, residuals)."""
    return _jacobi("spmdb200_jacobi2d", u, v, sweeps, res_every, ws, res, check, stream)


def jacobi3d(u: torch.Tensor, v: torch.Tensor, sweeps: int, res_every: int = 0, ws=None, res=None,
             check: bool = True, stream=None):
    """`sweeps` 7-point sweeps ping-ponging u -> v -> u ...; returns (final grid, residuals)."""
    return _jacobi("spmdb200_jacobi3d", u, v, sweeps, res_every, ws, res, check, stream)
