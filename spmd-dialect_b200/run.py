"""Command-line runner for one kernel family on one size -- the counterpart of
the reference's harness drivers with --perf (harness/run_ewise.py,
run_promoted_stencil.py, run_reduction.py): builds a seeded input on the
device, runs the kernel `--reps` times after `--warmup` runs and prints one
JSON line with the CUDA-event time per rep and the bandwidth it implies.

    python spmd-dialect_b200/run.py jacobi2d --shape 16384x16384 --sweeps 2 --reps 1
    python spmd-dialect_b200/run.py sum_f32 --size 16777216
    python spmd-dialect_b200/run.py jacobi3d --shape 512x512x512 --sweeps 4

Kernels: ewise, axpy, sum_f32, sum_i32, hierarchical_sum, stencil3, jacobi2d,
jacobi3d, reduce_f32 / reduce_i32 (--kind add|mul|max|min|and|or|xor), forall_map
(--body axpy: y = 2.5*x + y in place; --body 3in: r = sqrt(|a*b - c|)).  No checking
happens here (the parity tests compare against the
oracle); this is for timing and for profiler captures.
"""
from __future__ import annotations

import argparse
import importlib
import json
import statistics
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["ewise", "axpy", "sum_f32", "sum_i32", "hierarchical_sum", "stencil3",
                                       "stencil_nd", "jacobi2d", "jacobi3d", "reduce_f32", "reduce_i32", "forall_map"])
    ap.add_argument("--kind", default="max", help="reduction kind for reduce_f32 / reduce_i32")
    ap.add_argument("--body", default="3in", choices=["axpy", "3in"], help="forall_map body")
    ap.add_argument("--layout", default="vec", choices=["vec", "contig", "strided"],
                    help="forall_map views: 16-byte aligned, contiguous from element 1, or rows of 4096 in a "
                         "4097-element pitch")
    ap.add_argument("--size", type=int, default=1 << 24)
    ap.add_argument("--shape", default="4096x4096")
    ap.add_argument("--sweeps", type=int, default=100)
    ap.add_argument("--res-every", type=int, default=10)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--flush-l2", action="store_true", help="write 256 MiB between reps")
    a = ap.parse_args()

    import torch
    k = importlib.import_module("spmd-dialect_b200.kernels")
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(a.seed)
    shape = tuple(int(x) for x in a.shape.split("x"))
    work_bytes = 0
    updates = 0

    if a.kernel in ("ewise", "axpy"):
        x = torch.rand(a.size, device=dev, generator=g)
        y = torch.rand(a.size, device=dev, generator=g)
        out = torch.empty_like(x)
        fn = (lambda: k.ewise(x, y, out)) if a.kernel == "ewise" else (lambda: k.axpy(2.5, x, y))
        work_bytes = 12 * a.size
    elif a.kernel == "forall_map":
        fp = importlib.import_module("spmd-dialect_b200.forall_program")
        nv = 2 if a.body == "axpy" else 3

        def view(t):
            if a.layout == "contig":
                return t[1:a.size + 1]
            if a.layout == "strided":
                return t[: a.size // 4096 * 4097].view(-1, 4097)[:, :4096]
            return t[: a.size]

        alloc = a.size // 4096 * 4097 + 4097  # room for every layout
        xs = [view(torch.rand(alloc, device=dev, generator=g)) for _ in range(nv)]
        if a.body == "axpy":
            code, n_regs, _, _ = fp.compile_dag("s", {"x": ("load", 0), "y": ("load", 1), "a": ("const", 0),
                                                      "m": ("mul", "a", "x"), "s": ("add", "m", "y")})
            fn = lambda: k.forall_map(xs, xs[1], code, [2.5], n_regs=n_regs)  # noqa: E731
            work_bytes = 12 * a.size
        else:
            code, n_regs, _, _ = fp.compile_dag("r", {"a": ("load", 0), "b": ("load", 1), "c": ("load", 2),
                                                      "p": ("mul", "a", "b"), "d": ("sub", "p", "c"),
                                                      "q": ("abs", "d"), "r": ("sqrt", "q")})
            out = view(torch.empty(alloc, device=dev))
            fn = lambda: k.forall_map(xs, out, code, n_regs=n_regs)  # noqa: E731
            work_bytes = 16 * a.size
    elif a.kernel in ("sum_f32", "hierarchical_sum"):
        x = torch.rand(a.size, device=dev, generator=g)
        o = torch.zeros(1, device=dev)
        ws = k.sum_workspace(a.size)
        fn = (lambda: k.sum_f32(x, o, ws)) if a.kernel == "sum_f32" else (lambda: k.hierarchical_sum(x, o))
        work_bytes = 4 * a.size
    elif a.kernel == "sum_i32":
        x = torch.randint(0, 100, (a.size,), device=dev, dtype=torch.int32, generator=g)
        o = torch.zeros(1, device=dev, dtype=torch.int32)
        fn = lambda: k.sum_i32(x, o)  # noqa: E731
        work_bytes = 4 * a.size
    elif a.kernel in ("reduce_f32", "reduce_i32"):
        if a.kernel == "reduce_f32":
            x = torch.rand(a.size, device=dev, generator=g)
        else:
            x = torch.randint(-1000, 1000, (a.size,), device=dev, dtype=torch.int32, generator=g)
        ws = k.sum_workspace(a.size)
        o = torch.zeros(1, device=dev, dtype=x.dtype)
        fn = lambda: k.reduce(a.kind, x, 0, o, ws)  # noqa: E731
        work_bytes = 4 * a.size
    elif a.kernel == "stencil3":
        n, m = shape
        x = torch.rand((n + 1, m + 1), device=dev, generator=g)
        out = torch.empty((n, m), device=dev)
        fn = lambda: k.stencil3pt(x, out)  # noqa: E731
        work_bytes = 8 * n * m
    elif a.kernel == "stencil_nd":
        # The general promoted-tile stencil: the 5-point (rank 2) or 7-point
        # (rank 3) star in source order, scaled, output the size of the input.
        x = torch.rand(shape, device=dev, generator=g)
        out = torch.empty_like(x)
        r = len(shape)
        taps = [[0] * r]
        for d in range(r):
            for o in (-1, 1):
                t = [0] * r
                t[d] = o
                taps.append(t)
        fn = lambda: k.stencil_nd(x, out, taps, scale=1.0 / len(taps))  # noqa: E731
        work_bytes = 8 * x.numel()
    else:
        u = torch.rand(shape, device=dev, generator=g)
        v = torch.empty_like(u)
        ws = k.jacobi_workspace()
        nres = a.sweeps // a.res_every if a.res_every > 0 else 0
        res = torch.zeros(max(nres, 1), dtype=torch.float64, device=dev)
        run = k.jacobi2d if a.kernel == "jacobi2d" else k.jacobi3d
        fn = lambda: run(u, v, a.sweeps, a.res_every, ws=ws, res=res, check=False)  # noqa: E731
        cells = 1
        for s in shape:
            cells *= s
        updates = cells * a.sweeps
        work_bytes = 8 * updates

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if a.flush_l2 else None
    st = torch.cuda.current_stream()
    for _ in range(a.warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(a.reps):
        if flush is not None:
            flush.zero_()
        torch.cuda._sleep(200_000)  # keep the stream busy so launch latency stays out of the interval
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        fn()
        e1.record(st)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    if a.kernel in ("jacobi2d", "jacobi3d"):
        k.workspace_status(ws)
    ms = statistics.median(ts)
    line = {"kernel": a.kernel, "ms": round(ms, 5), "reps": a.reps, "GB/s": round(work_bytes / ms / 1e6, 1)}
    if updates:
        line["Gcell/s"] = round(updates / ms / 1e6, 2)
        line["shape"] = list(shape)
        line["sweeps"] = a.sweeps
    else:
        line["size"] = a.size
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
