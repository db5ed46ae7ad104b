"""1-D operations split across GPUs, one process per GPU.

The reductions and the elementwise forall shard trivially: every rank owns a
contiguous block of the N elements (shard_range) and runs the single-GPU
kernel on it.

* sum_f32: each rank computes the unrounded f64 total of its block
  (spmdb200_sum_f32_partial), the partials are all-gathered and added in rank
  order on the host, and the single f32 rounding of init + total happens
  once -- the same value on every rank, independent of NCCL's reduction
  order.
* sum_i32: the per-rank totals are combined exactly (int64 all-reduce) and
  wrapped to int32, which equals the single-GPU wrapping sum.
* axpy: y = a*x + y needs no exchange at all.

torch.distributed (NCCL on GPUs, gloo in the CPU tests) carries the partials.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import c_i, c_p, call


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of `rank`'s contiguous block of n elements (sizes differ by at most 1)."""
    if not (0 <= rank < world) or n < 0:
        raise ValueError(f"rank {rank} of {world}, n = {n}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def combine_f32(partials, init: float = 0.0) -> np.float32:
    """f32(f64(init) + p0 + p1 + ...) with the partials added in rank order."""
    tot = 0.0
    for p in partials:
        tot = tot + float(p)
    return np.float32(float(np.float32(init)) + tot)


def combine_i32(totals, init: int = 0) -> int:
    """Wrapping int32 sum of init and the per-rank totals."""
    t = (int(init) + sum(int(x) for x in totals)) & 0xFFFFFFFF
    return t - (1 << 32) if t >= (1 << 31) else t


def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() else None


def partial_sum_f32(x, ws=None, stream=None):
    """Device f64 scalar tensor: the unrounded total of this rank's block."""
    import torch

    from .kernels import memref, sum_workspace
    n = x.shape[0]
    ws = sum_workspace(n, x.device) if ws is None else ws
    out = torch.empty(1, dtype=torch.float64, device=x.device)
    s = torch.cuda.current_stream() if stream is None else stream
    call("spmdb200_sum_f32_partial", *memref(x), c_i(n), c_p(out.data_ptr()), c_p(ws.data_ptr()),
         ctypes.c_size_t(ws.numel()), c_p(s.cuda_stream))
    return out


def sum_f32(x_local, init: float = 0.0, ws=None) -> np.float32:
    """Sum over every rank's block; the same f32 on every rank."""
    import torch
    d = _dist()
    p = partial_sum_f32(x_local, ws)
    world = d.get_world_size() if d else 1
    if world == 1:
        return combine_f32([float(p.item())], init)
    parts = [torch.empty_like(p) for _ in range(world)]
    d.all_gather(parts, p)
    return combine_f32([float(t.item()) for t in parts], init)


def sum_i32(x_local, init: int = 0) -> int:
    """Exact wrapping int32 sum over every rank's block; the same on every rank."""
    import torch

    from .kernels import sum_i32 as local_sum
    d = _dist()
    out = torch.zeros(1, dtype=torch.int32, device=x_local.device)
    local_sum(x_local, out)
    tot = out.to(torch.int64)
    if d is not None and d.get_world_size() > 1:
        d.all_reduce(tot)
    return combine_i32([int(tot.item())], init)


def axpy(alpha: float, x_local, y_local):
    """y = a*x + y on this rank's block (no exchange)."""
    from .kernels import axpy as local_axpy
    return local_axpy(alpha, x_local, y_local)
