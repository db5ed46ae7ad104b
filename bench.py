"""Benchmark: Jacobi-2D Gcell-updates/s (+ reduction GB/s) and % of HBM roofline on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl spmd|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

Workload (one "step"): the multi-GPU Jacobi-2D configuration -- a 32768 x 32768
f32 row slab per GPU (weak scaling: the global grid is (32768*N) x 32768),
interior uniform [0,1) from seed 4, zero boundary rows/columns, 1000 ping-pong
sweeps, a global L2 residual every 10 sweeps.  Inputs are device-resident when
the timed region starts (4 GiB per grid, far above the 126 MB L2, so no L2
flush is needed between steps).  At N > 1 the slabs exchange eight halo rows per
neighbour per pass over NVLink inside the persistent kernel.

`value` is device time (CUDA events, max over ranks); `e2e` runs the same job
through the host-buffer C entries (pinned host grids in, result grids out,
every copy inside the timed region).  `roofline` uses the algorithmic bytes of
the sweep kernel against the measured HBM copy bandwidth: each pass over the
grid reads every cell once and writes it once (8 B per cell per pass), and a
pass advances eight sweeps (1000 sweeps with a residual every 10: 124 passes
of eight and 2 of four), so 1000 sweeps cost 1.008 B per cell update.

Before anything is timed the run checks its own results (`parity`, and a
non-zero exit on any mismatch): at N = 1 the timed kernel on a 2048 x 32768
slab of RandomState(4) input for the full 1000 sweeps against the oracle; at
N > 1 a gathered row-slab grid and a gathered z-slab grid against the
single-domain oracle, and the sharded sums against the f64 sum.

At N > 1 the line also carries the configured global grid split across the
GPUs (`strong`: 32768 x 32768 in 32768/N-row slabs), the sharded f32/i32 sums
(2^24 elements per GPU) and the Jacobi-3D z-slab run (512^3 per GPU).

`cpu_baseline` times the oracle (the C/OpenMP restatement of the reference's
SPMDToOpenMP lowering) on a bounded sample of the same grid, on every host core
(set explicitly: launchers export OMP_NUM_THREADS=1), before torch is loaded.
`--impl reference` times that CPU path alone (the reference itself needs
MLIR/LLVM 20 to build and cannot run here).
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Jacobi-2D Gcell-updates/s & reduction GB/s, % of HBM roofline, at 1/2/4/8 B200"
GRID = 32768
SWEEPS = 1000
RES_EVERY = 10
BYTES_PER_CELL_PASS = 8  # algorithmic: each pass reads u[i,j] once and writes v[i,j] once
J3_FMAX = 2  # longest Jacobi-3D pass (sweeps), = the 3-D z-slab halo depth the library reports
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) over algorithmic bytes of the dominant Jacobi-2D
# kernel, measured by ncu (--set full) on a 16384^2 grid in two eight-sweep
# passes: 4.626 GB for 4.295e9 updates at 1.0 algorithmic B/update.  The
# benchmark grid is too large for a multi-pass capture; traffic grows with
# cells x passes, so a launch's traffic is this ratio x its algorithmic bytes.
TRAFFIC_OVER_ALGORITHMIC = {"jacobi2d_wave_kernel<8>": 1.077}
# Parity slab of the headline kernel: rows x columns of RandomState(4) input.
PARITY_ROWS = 2048


def sweep_passes(sweeps: int, res_every: int, fmax: int = 8) -> dict[int, int]:
    """{sweeps per pass: passes} as the Jacobi kernels schedule them: even
    numbers of 8- (2-D only), 4- and 2-sweep passes (none longer than the
    residual interval), then the single sweeps left over.  fmax: 8 for the
    2-D kernel, J3_FMAX for the 3-D one."""
    top = fmax
    while res_every > 0 and fmax > res_every:
        fmax //= 2
    plan, left = {}, sweeps
    for f in [x for x in (8, 4, 2, 1) if x <= top]:
        n = 0 if f > fmax else left if f == 1 else (left // (2 * f)) * 2
        plan[f] = n
        left -= n * f
    return plan


def bytes_per_update(sweeps: int, res_every: int, fmax: int = 8) -> float:
    return BYTES_PER_CELL_PASS * sum(sweep_passes(sweeps, res_every, fmax).values()) / sweeps


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def jacobi_init(shape, seed: int) -> np.ndarray:
    """Interior uniform [0,1) from RandomState(seed), boundary cells 0."""
    u = np.random.RandomState(seed).random_sample(shape).astype(np.float32)
    if u.ndim == 2:
        u[0, :] = 0; u[-1, :] = 0; u[:, 0] = 0; u[:, -1] = 0
    else:
        u[0] = 0; u[-1] = 0; u[:, 0] = 0; u[:, -1] = 0; u[:, :, 0] = 0; u[:, :, -1] = 0
    return u


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def max_rel(a: np.ndarray, b: np.ndarray) -> float:
    if b.size == 0:
        return 0.0
    return float(np.max(np.abs(np.asarray(a) - b) / np.maximum(np.abs(b), 1e-300)))


# ------------------------------------------------------------------ clocks sampler
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread:
                self.thread.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        under_load = [s for s in sm if s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(under_load), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ distributed plumbing
def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ CPU (oracle) legs
def cpu_jacobi_sample(target_s: float = 12.0, rows: int = 2048, cols: int = GRID) -> dict:
    """Oracle Jacobi-2D sweeps over a rows x cols slab of the workload grid (same
    row width) on every host core, repeated until ~target_s of CPU work;
    Gcell-updates/s."""
    from oracle import oracle
    threads = oracle.set_num_threads(cpu_count())
    u = jacobi_init((rows, cols), 4)
    v = np.empty_like(u)
    rr = np.zeros(rows, np.float64)
    for _ in range(2):  # warm-up (page faults, thread pool)
        oracle.jacobi2d_rows(u, v, 0, rows, 0, rows)
    sweeps, t0 = 0, time.perf_counter()
    while True:
        want = (sweeps + 1) % RES_EVERY == 0
        oracle.lib().oracle_jacobi2d_rows(oracle._p(u), oracle._p(v), cols, cols, 0, rows, 0, rows,
                                          oracle._p(rr) if want else None)
        u, v = v, u
        sweeps += 1
        el = time.perf_counter() - t0
        if el >= target_s and sweeps >= 3:
            break
    gcell = rows * cols * sweeps / el / 1e9
    return {"value": round(gcell, 4), "unit": "Gcell-updates/s", "cores": threads, "kind": "port",
            "sample": f"{rows}x{cols} rows of the workload grid, {sweeps} sweeps (residual every {RES_EVERY}), "
                      f"{el:.1f} s, OpenMP threads={threads} (set explicitly), host cpus={cpu_count()}"}


def oracle_headline_parity() -> tuple[np.ndarray, np.ndarray, np.ndarray, float]:
    """(input, oracle grid, oracle residuals, seconds) of the headline kernel's
    parity case: a PARITY_ROWS x 32768 RandomState(4) slab, 1000 sweeps,
    residual every 10."""
    from oracle import oracle
    oracle.set_num_threads(cpu_count())
    u0 = jacobi_init((PARITY_ROWS, GRID), 4)
    t0 = time.perf_counter()
    want, wres = oracle.jacobi2d(u0, SWEEPS, RES_EVERY)
    return u0, want, wres, time.perf_counter() - t0


def run_reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    # Each step: a bounded sample of the workload on all host cores.
    for _ in range(args.warmup):
        cpu_jacobi_sample(target_s=2.0)
    vals, times = [], []
    r = None
    for _ in range(args.steps):
        t0 = time.perf_counter()
        r = cpu_jacobi_sample(target_s=6.0)
        times.append((time.perf_counter() - t0) * 1e3)
        vals.append(r["value"])
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Gcell-updates/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.mean(times), 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic: RandomState(4) uniform [0,1), zero boundary",
        "config": {"workload": "jacobi2d 5-point, 32768 columns x 2048-row sample, 1000-sweep config, CPU",
                   "grid": [GRID, GRID], "sweeps": SWEEPS, "res_every": RES_EVERY},
        "cpu_baseline": {**r, "value": value},
        "e2e": {"value": value, "unit": "Gcell-updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's SPMDToOpenMP path needs MLIR/LLVM 20.1.7 to build (absent, no network); "
                "this arm times the C/OpenMP restatement of that lowering (the oracle) on all host cores",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU legs
def refabi_benchmarks(torch, hbm_peak: float) -> dict:
    """The reference-named kernels of spmdb200_kernels.cubin, loaded with
    cuModuleLoadData and launched with the reference harness's own launch
    shapes, sizes and timing methods: ewise_kernel (tile 32, N = 1e7, wall
    clock per launch over 20 asynchronous launches, harness/run_ewise.py:127-132),
    promoted_stencil_kernel (32 x 8 tile, 297 threads, 4096^2, wall clock over 10
    launches, harness/run_promoted_stencil.py:184-188) and
    hierarchical_sum_kernel (tile 256, 2^24, CUDA events around each launch
    after a memset of the output, mean of 10, harness/run_reduction.py:307-315)."""
    cd = importlib.import_module("spmd-dialect_b200.cuda_driver")
    lib_mod = importlib.import_module("spmd-dialect_b200._lib")
    cd.init(torch.cuda.current_device())
    mod = cd.load_cubin(str(lib_mod.CUBIN_PATH))
    out = {}
    rng = np.random.default_rng(0)

    def wall(launch, reps):
        for _ in range(3):
            launch()
        cd.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            launch()
        cd.synchronize()
        return (time.perf_counter() - t0) / reps * 1e3

    n = 10_000_000
    a = rng.random(n, dtype=np.float32)
    b = rng.random(n, dtype=np.float32)
    ad, bd, cdv = cd.alloc(a.nbytes), cd.alloc(b.nbytes), cd.alloc(a.nbytes)
    cd.memcpy_h2d(ad, a)
    cd.memcpy_h2d(bd, b)
    fn = cd.get_function(mod, "ewise_kernel")
    tile = 32
    ms = wall(lambda: cd.launch(fn, (math.ceil(n / tile), 1, 1), (tile, 1, 1), tile, n, ad, ad, 0, n, 1,
                                bd, bd, 0, n, 1, cdv, cdv, 0, n, 1), 20)
    c = np.empty(n, np.float32)
    cd.memcpy_d2h(c, cdv)
    for p in (ad, bd, cdv):
        p.free()
    gbs = n * 12 / ms / 1e6
    out["ewise_kernel_1e7"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3),
                               "reference_ms": 0.206, "launch": "grid ceil(N/32), block 32",
                               "timing": "wall clock per launch, 20 async launches (run_ewise.py)",
                               "max_abs_err": float(np.max(np.abs(c - (a + b))))}
    N = M = 4096
    tr, tc = 32, 8
    a = rng.random((N, M), dtype=np.float32)
    ad, bd = cd.alloc(a.nbytes), cd.alloc(a.nbytes)
    cd.memcpy_h2d(ad, a)
    fn = cd.get_function(mod, "promoted_stencil_kernel")
    grid = (math.ceil(N / tr), math.ceil(M / tc), 1)
    ms = wall(lambda: cd.launch(fn, grid, ((tr + 1) * (tc + 1), 1, 1), tr, tc, ad, ad, 0, N, M, M, 1, 1,
                                bd, bd, 0, N, M, M, 1), 10)
    bh = np.zeros((N, M), np.float32)
    cd.memcpy_d2h(bh, bd)
    ad.free()
    bd.free()
    ref = a[:-1, :-1] + a[:-1, 1:] + a[1:, :-1]
    gbs = 2 * N * M * 4 / ms / 1e6
    out["promoted_stencil_kernel_4096^2"] = {
        "ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3), "reference_ms": 0.285,
        "launch": "grid (128, 512), block 297 (33 x 9)", "timing": "wall clock per launch, 10 async launches "
        "(run_promoted_stencil.py)", "max_abs_err": float(np.max(np.abs(bh[:-1, :-1] - ref)))}
    n = 1 << 24
    a = rng.random(n, dtype=np.float32)
    ad, od = cd.alloc(a.nbytes), cd.alloc(4)
    cd.memcpy_h2d(ad, a)
    fn = cd.get_function(mod, "hierarchical_sum_kernel")
    e0, e1 = cd.event_create(), cd.event_create()
    for _ in range(3):
        cd.memset(od, 0, 4)
        cd.launch(fn, (n // 256, 1, 1), (256, 1, 1), 256, n, ad, od)
    cd.synchronize()
    tot = 0.0
    for _ in range(10):
        cd.memset(od, 0, 4)
        cd.event_record(e0)
        cd.launch(fn, (n // 256, 1, 1), (256, 1, 1), 256, n, ad, od)
        cd.event_record(e1)
        tot += cd.event_elapsed_ms(e0, e1)
    ms = tot / 10
    r = np.zeros(1, np.float32)
    cd.memcpy_d2h(r, od)
    cd.event_destroy(e0)
    cd.event_destroy(e1)
    ad.free()
    od.free()
    f64 = float(np.sum(a.astype(np.float64)))
    gbs = n * 4 / ms / 1e6
    out["hierarchical_sum_kernel_2^24"] = {
        "ms": round(ms, 5), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3), "reference_ms": 0.112,
        "launch": "grid 65536, block 256", "timing": "CUDA events per launch, mean of 10 (run_reduction.py)",
        "rel_err_vs_f64": abs(float(r[0]) - f64) / f64, "l2": "input may be L2-resident, as in the reference's run"}
    return out


def secondary_benchmarks(kernels, torch, hbm_peak: float) -> dict:
    """The other configurations at N=1 (rank 0): f32/i32 sum 2^24, f32 max and
    i32 xor reductions 2^24, axpy 2^28,
    the promoted 3-point stencil at 4096^2 and 8192^2, the general stencil
    (5-point) at 8192^2, Jacobi-2D 4096^2 x 100, Jacobi-3D 512^3 x 50, and the
    reference-named kernels at the reference's launch shapes.  L2 flushed
    between reps unless stated."""
    out = {}
    dev = torch.device("cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MiB > 126 MB L2
    st = torch.cuda.current_stream()

    def timed(fn, reps=10, warm=3, flush_l2=True):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(reps):
            if flush_l2:
                flush.zero_()
            torch.cuda._sleep(200_000)  # busy stream: the host's launch latency stays outside the interval
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            fn()
            b.record(st)
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    # Reductions: 2^24 elements (64 MiB) is below the 126 MB L2, so consecutive
    # launches read different ones of 4 copies (256 MiB rotation): every read
    # comes from HBM and no flush write-back is charged to the kernel.  Two
    # figures: one launch between two events (the stream kept busy so the
    # host's launch latency stays outside), and the mean of 40 back-to-back
    # launches (programmatic dependent launch overlaps each prologue with the
    # previous kernel's tail).
    def batch(fn_i, n_launch=40):
        for i in range(3):
            fn_i(i)
        torch.cuda.synchronize()
        torch.cuda._sleep(2_000_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for i in range(n_launch):
            fn_i(i)
        b.record(st)
        b.synchronize()
        return a.elapsed_time(b) / n_launch

    g = torch.Generator(device=dev).manual_seed(0)
    n = 1 << 24
    bufs = [torch.rand(n, device=dev, generator=g) for _ in range(4)]
    ibufs = [torch.randint(0, 100, (n,), device=dev, dtype=torch.int32, generator=g) for _ in range(4)]
    o = torch.zeros(1, device=dev)
    oi = torch.zeros(1, device=dev, dtype=torch.int32)
    ws = kernels.sum_workspace(n)
    # sum_f32: the deterministic sum (one f32 rounding, identical bits on every
    # call); hierarchical_sum_f32: the reference's own semantics (one f32
    # atomic per block, SPMDToGPU.cpp's grid combine), no last-block combine.
    for key, fn_i in (("sum_f32_2^24", lambda i: kernels.sum_f32(bufs[i % 4], o, ws)),
                      ("hierarchical_sum_f32_2^24", lambda i: kernels.hierarchical_sum(bufs[i % 4], o)),
                      ("sum_i32_2^24", lambda i: kernels.sum_i32(ibufs[i % 4], oi))):
        ms = batch(fn_i)
        it = iter(range(1 << 30))
        ms1 = timed(lambda: fn_i(next(it)), reps=20, flush_l2=False)
        gbs = n * 4 / ms / 1e6
        out[key] = {"ms": round(ms, 5), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3),
                    "ms_single_launch": round(ms1, 5),
                    "frac_of_hbm_single_launch": round(n * 4 / ms1 / 1e6 / hbm_peak, 3),
                    "l2": "4 rotating 64 MiB inputs", "timing": "mean of 40 back-to-back launches; single launch: "
                    "median of 20, CUDA events around one launch"}
    # The single-launch method's own floor: an empty kernel between the same
    # two events (the reductions' single-launch times include it).
    out["single_launch_floor"] = {"ms_empty_kernel": round(timed(lambda: torch.cuda._sleep(0), reps=20,
                                                                 flush_l2=False), 5),
                                  "ms_sum_f32_4096_elements": round(timed(lambda: kernels.sum_f32(bufs[0][:4096], o, ws),
                                                                          reps=20, flush_l2=False), 5)}
    # Other spmd.reduce kinds on the same inputs (f32 max: integer max over
    # order-preserving keys; i32 xor), same timing.
    ok_ = torch.zeros(1, device=dev)
    oki = torch.zeros(1, device=dev, dtype=torch.int32)
    for key, fn_i in (("reduce_max_f32_2^24", lambda i: kernels.reduce("max", bufs[i % 4], 0.0, ok_, ws)),
                      ("reduce_xor_i32_2^24", lambda i: kernels.reduce("xor", ibufs[i % 4], 0, oki, ws))):
        ms = batch(fn_i)
        gbs = n * 4 / ms / 1e6
        out[key] = {"ms": round(ms, 5), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3),
                    "l2": "4 rotating 64 MiB inputs", "timing": "mean of 40 back-to-back launches"}
    del bufs, ibufs
    n = 1 << 28
    x = torch.rand(n, device=dev, generator=g) * 2 - 1
    y = torch.rand(n, device=dev, generator=g) * 2 - 1
    ms = timed(lambda: kernels.axpy(2.5, x, y), flush_l2=False)
    gbs = n * 12 / ms / 1e6
    out["axpy_2^28"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3)}
    # The general elementwise forall (body program in shared-memory registers)
    # on the same axpy body, and on a three-input body sqrt(|a*b - c|).
    fp = importlib.import_module("spmd-dialect_b200.forall_program")
    ax = fp.compile_dag("s", {"x": ("load", 0), "y": ("load", 1), "a": ("const", 0), "m": ("mul", "a", "x"),
                              "s": ("add", "m", "y")})
    ms = timed(lambda: kernels.forall_map([x, y], y, ax[0], [2.5], n_regs=ax[1]), flush_l2=False)
    gbs = n * 12 / ms / 1e6
    out["forall_map_axpy_body_2^28"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1),
                                        "frac_of_hbm": round(gbs / hbm_peak, 3), "insns": len(ax[0])}
    z = torch.empty_like(x)
    b3 = fp.compile_dag("r", {"a": ("load", 0), "b": ("load", 1), "c": ("load", 2), "p": ("mul", "a", "b"),
                              "d": ("sub", "p", "c"), "q": ("abs", "d"), "r": ("sqrt", "q")})
    n3 = n // 2
    xs, ys, zs = x[:n3], y[:n3], y[n3:]
    ms = timed(lambda: kernels.forall_map([xs, ys, zs], z[:n3], b3[0], n_regs=b3[1]), flush_l2=False)
    gbs = n3 * 16 / ms / 1e6
    out["forall_map_3in_2^27"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3),
                                  "insns": len(b3[0])}
    del x, y, z
    # Promoted 3-point stencil B = (A + A east) + A south on the harness layout
    # (A is (N+1) x (N+1)): 4096^2 is the reference's own configuration, 8192^2
    # the same above the L2 size.  Bytes: A read once, B written once.
    for nn in (4096, 8192):
        a = torch.rand((nn + 1, nn + 1), device=dev, generator=g)
        b = torch.empty((nn, nn), device=dev)
        ms = timed(lambda: kernels.stencil3pt(a, b))
        gbs = (a.numel() + b.numel()) * 4 / ms / 1e6
        out[f"stencil3pt_{nn}^2"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1),
                                     "frac_of_hbm": round(gbs / hbm_peak, 3)}
        del a, b
    # General promoted-tile stencil: Jacobi-2D 5-point, one sweep, 8192^2.
    a = torch.rand((8192, 8192), device=dev, generator=g)
    b = torch.empty_like(a)
    j5 = [[0, 0], [-1, 0], [1, 0], [0, 1], [0, -1]]
    ms = timed(lambda: kernels.stencil_nd(a, b, j5, scale=0.2, tile_sizes=[16, 32]))
    gbs = 2 * a.numel() * 4 / ms / 1e6
    out["stencil_nd_5pt_8192^2"] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_peak, 3)}
    del a, b
    u = torch.rand((4096, 4096), device=dev, generator=g)
    u[0] = 0; u[-1] = 0; u[:, 0] = 0; u[:, -1] = 0
    v = torch.empty_like(u)
    jws = kernels.jacobi_workspace()
    res = torch.zeros(10, dtype=torch.float64, device=dev)
    ms = timed(lambda: kernels.jacobi2d(u, v, 100, 10, ws=jws, res=res, check=False), reps=5)
    kernels.workspace_status(jws)
    gc = 4096 * 4096 * 100 / ms / 1e6
    out["jacobi2d_4096^2_x100"] = {"ms": round(ms, 4), "Gcell/s": round(gc, 1),
                                   "frac_of_hbm": round(gc * bytes_per_update(100, 10) / hbm_peak, 3),
                                   "note": "128 MiB working set is L2-sized: fractions above 1 mean L2 reuse"}
    del u, v
    u = torch.rand((512, 512, 512), device=dev, generator=g)
    v = torch.empty_like(u)
    res = torch.zeros(5, dtype=torch.float64, device=dev)
    ms = timed(lambda: kernels.jacobi3d(u, v, 50, 10, ws=jws, res=res, check=False), reps=3, warm=1)
    kernels.workspace_status(jws)
    gc = 512 ** 3 * 50 / ms / 1e6
    out["jacobi3d_512^3_x50"] = {"ms": round(ms, 3), "Gcell/s": round(gc, 1),
                                 "passes": sweep_passes(50, 10, J3_FMAX),
                                 "frac_of_hbm": round(gc * bytes_per_update(50, 10, J3_FMAX) / hbm_peak, 3)}
    del u, v, flush
    torch.cuda.empty_cache()
    out.update(refabi_benchmarks(torch, hbm_peak))
    return out


def headline_parity(kernels, torch, dev, u0, want, wres) -> dict:
    """The timed kernel (same path, same row width, same 126 passes of eight and four sweeps)
    on the PARITY_ROWS x 32768 slab against the oracle."""
    u = torch.from_numpy(u0).to(dev)
    v = torch.empty_like(u)
    fin, res = kernels.jacobi2d(u, v, SWEEPS, RES_EVERY)
    got = fin.cpu().numpy()
    gres = res.cpu().numpy()
    bit_exact = same_bits(got, want)
    rel = max_rel(gres, wres)
    return {"case": f"{PARITY_ROWS}x{GRID} RandomState(4), {SWEEPS} sweeps, residual every {RES_EVERY}",
            "bit_exact": bit_exact, "residual_max_rel": rel, "ok": bool(bit_exact and rel <= 1e-12)}


def slab_parity(slab, torch, dist, rank: int, world: int) -> dict:
    """Row slabs and z-slabs across the ranks, gathered on rank 0 and compared
    with the single-domain oracle: an uneven row split that runs two- and
    one-sweep passes (residual every 3) and one that runs eight- and four-sweep
    passes (residual every 8), and an uneven plane split."""
    out = {}
    ok = torch.zeros(1, dtype=torch.int32, device="cuda")
    cases_ok = True
    for name, (G, W, runs, res_every) in (("slab2d", (64 * world + 5, 4100, (13,), 3)),
                                          ("slab2d_deep", (200 * world + 3, 3001, (28, 9), 8))):
        u0 = jacobi_init((G, W), 4)
        job = slab.SlabJacobi2D(cols=W, G=G, res_every=res_every, init=u0)
        for n in runs:  # back to back, no host synchronisation between the runs
            job.run(n, check=False)
        job.check()
        res = job.residuals()
        grid = job.gather()
        job.close()
        if rank == 0:
            from oracle import oracle
            want, _ = oracle.jacobi2d(u0, sum(runs), 0)
            _, wres = oracle.jacobi2d(jacobi_init((G, W), 4) if len(runs) == 1 else
                                      oracle.jacobi2d(u0, sum(runs[:-1]), 0)[0], runs[-1], res_every)
            be, rel = same_bits(grid, want), max_rel(res, wres)
            out[name] = {"case": f"{G}x{W} over {world} ranks, runs of {list(runs)} sweeps, residual every "
                                 f"{res_every}", "bit_exact": be, "residual_max_rel": rel,
                         "ok": bool(be and rel <= 1e-12)}
            cases_ok = cases_ok and out[name]["ok"]
    D, H, W3, sweeps3, res3 = 8 * world + 3, 36, 130, 7, 2
    u0 = jacobi_init((D, H, W3), 3)
    job = slab.SlabJacobi3D(H=H, W=W3, D=D, res_every=res3, init=u0)
    job.run(sweeps3)
    res = job.residuals()
    grid = job.gather()
    job.close()
    if rank == 0:
        from oracle import oracle
        want, wres = oracle.jacobi3d(u0, sweeps3, res3)
        be, rel = same_bits(grid, want), max_rel(res, wres)
        out["slab3d"] = {"case": f"{D}x{H}x{W3} over {world} ranks, {sweeps3} sweeps, residual every {res3}",
                         "bit_exact": be, "residual_max_rel": rel, "ok": bool(be and rel <= 1e-12)}
        ok.fill_(int(cases_ok and out["slab3d"]["ok"]))
    dist.broadcast(ok, 0)
    return out


def timed_steps(step, steps: int, warmup: int, world: int, dist, torch, finish=None,
                region=None) -> tuple[float, float]:
    """(ms per step over the whole timed region, mean per-step event time), max
    over ranks; W untimed steps first, barrier + synchronize on both sides.
    `region` (a context manager, e.g. the clock sampler) brackets the timed
    steps only."""
    import contextlib
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        step()
    if finish:
        finish()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    with region if region is not None else contextlib.nullcontext():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        evs[0].record(stream)
        for k in range(steps):
            step()
            evs[k + 1].record(stream)
        torch.cuda.synchronize()
    if finish:
        finish()
    per_step = [evs[k].elapsed_time(evs[k + 1]) for k in range(steps)]
    t = torch.tensor([evs[0].elapsed_time(evs[-1]) / steps, statistics.mean(per_step)], dtype=torch.float64,
                     device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0]), float(t[1])


def multi_gpu_records(slab, shard, kernels, torch, dist, rank: int, world: int, args, hbm_peak: float) -> dict:
    """N > 1: the configured 32768^2 global grid split over the ranks (strong
    scaling), the sharded sums at 2^24 elements per GPU, and Jacobi-3D z-slabs
    at 512^3 per GPU."""
    out = {}
    steps, warm = max(3, args.steps), 3
    # ---- strong: 32768 x 32768 global, 32768/N rows per rank
    job = slab.SlabJacobi2D(cols=GRID, G=GRID, seed=4, res_every=RES_EVERY)
    ms, _ = timed_steps(lambda: job.run(SWEEPS, check=False), steps, warm, world, dist, torch, job.check)
    job.close()
    out["strong"] = {"workload": "jacobi2d 32768x32768 global (the configured grid) in 32768/N-row slabs, "
                                 "1000 sweeps, residual every 10",
                     "value": round(GRID * GRID * SWEEPS / (ms * 1e-3) / 1e9, 3), "unit": "Gcell-updates/s",
                     "ms_per_step": round(ms, 3), "rows_per_rank": GRID // world, "steps": steps}
    # ---- sharded sums: 2^24 elements per rank (weak), one all-gather / all-reduce
    n = 1 << 24
    rs = np.random.RandomState(100 + rank)
    xf = torch.from_numpy(rs.random_sample(n).astype(np.float32)).cuda()
    xi = torch.from_numpy(rs.randint(0, 100, n).astype(np.int32)).cuda()
    local64 = torch.tensor([float(np.sum(xf.cpu().numpy().astype(np.float64))),
                            float(xi.cpu().numpy().astype(np.int64).sum())], dtype=torch.float64, device="cuda")
    dist.all_reduce(local64)
    ws = kernels.sum_workspace(n)
    got_f = shard.sum_f32(xf, ws=ws)
    got_i = shard.sum_i32(xi)
    exact_f, exact_i = float(local64[0]), int(local64[1])
    ok_f = abs(float(got_f) - exact_f) <= 1e-6 * exact_f
    ok_i = got_i == shard.combine_i32([exact_i])  # the int32 wrap of the exact total
    stream = torch.cuda.current_stream()
    oi = torch.zeros(1, dtype=torch.int32, device="cuda")

    def med_ms(fn, reps=20, hide_launch=False):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ts = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if hide_launch:
                torch.cuda._sleep(200_000)  # busy stream: the host's launch latency stays outside the interval
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            ts.append(a.elapsed_time(b))
        t = torch.tensor([statistics.median(ts)], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    recs = {}
    for key, fn, local_fn in (("sum_f32", lambda: shard.sum_f32(xf, ws=ws), lambda: shard.partial_sum_f32(xf, ws)),
                              ("sum_i32", lambda: shard.sum_i32(xi), lambda: kernels.sum_i32(xi, oi))):
        ms = med_ms(fn)  # local kernel + NCCL exchange + the host read of the combined result
        ms_k = med_ms(local_fn, hide_launch=True)  # this rank's kernel alone
        recs[key] = {"ms": round(ms, 5), "GB/s_total": round(world * n * 4 / ms / 1e6, 1),
                     "ms_local_kernel": round(ms_k, 5),
                     "GB/s_per_gpu_kernel": round(n * 4 / ms_k / 1e6, 1),
                     "frac_of_hbm_per_gpu_kernel": round(n * 4 / ms_k / 1e6 / hbm_peak, 3)}
    out["sharded_sums"] = {"elements_per_gpu": n, **recs,
                           "timing": "CUDA events around one sharded sum (local kernel, NCCL exchange, host "
                                     "combine) and around the local kernel alone (launch latency hidden behind "
                                     "a busy stream), median of 20, max over ranks",
                           "f32_rel_err_vs_f64": abs(float(got_f) - exact_f) / exact_f, "f32_ok": bool(ok_f),
                           "i32_exact": bool(ok_i)}
    # ---- Jacobi-3D z-slabs, 512^3 per rank (weak)
    job3 = slab.SlabJacobi3D(H=512, W=512, planes_per_rank=512, seed=3, res_every=10)
    ms3, _ = timed_steps(lambda: job3.run(50, check=False), steps, warm, world, dist, torch, job3.check)
    job3.close()
    out["jacobi3d_slab"] = {"workload": "jacobi3d 7-point, 512^3 per GPU in z-slabs (global 512N x 512 x 512), "
                                        "50 sweeps, residual every 10",
                            "value": round(world * 512 ** 3 * 50 / (ms3 * 1e-3) / 1e9, 3),
                            "unit": "Gcell-updates/s", "ms_per_step": round(ms3, 3), "steps": steps}
    return out, bool(ok_f and ok_i)


def run_spmd_arm(args) -> None:
    rank, world, local = dist_env()
    # ---- CPU work first, before torch is loaded: torch brings its own OpenMP
    # pool, whose spinning threads would compete with the oracle's.
    cpu = None
    headline_case = None
    if rank == 0 and world == 1:
        cpu = cpu_jacobi_sample()
        headline_case = oracle_headline_parity()

    import torch
    import torch.distributed as dist

    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    kernels = importlib.import_module("spmd-dialect_b200.kernels")
    halo3 = int(importlib.import_module("spmd-dialect_b200._lib").lib().spmdb200_jacobi_slab_halo(3))
    if halo3 != J3_FMAX:
        raise RuntimeError(f"the library's 3-D passes are up to {halo3} sweeps, bench.py assumes {J3_FMAX}")
    slab = importlib.import_module("spmd-dialect_b200.slab") if world > 1 else None
    shard = importlib.import_module("spmd-dialect_b200.shard") if world > 1 else None
    hbm_peak, peak_kind = measured_peaks()

    # ---- parity of what is about to be timed -----------------------------------
    parity = {}
    if world == 1:
        u0, want, wres, oracle_s = headline_case
        parity["jacobi2d"] = {**headline_parity(kernels, torch, dev, u0, want, wres),
                              "oracle_s": round(oracle_s, 1)}
        del u0, want, wres, headline_case
        parity_ok = parity["jacobi2d"]["ok"]
    else:
        parity = slab_parity(slab, torch, dist, rank, world)
        flag = torch.tensor([1 if (rank != 0 or all(p["ok"] for p in parity.values())) else 0],
                            dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        parity_ok = bool(flag.item())

    # ---- device-resident workload ------------------------------------------------
    rows = GRID
    if world == 1:
        g = torch.Generator(device=dev).manual_seed(4)
        u = torch.rand((rows, GRID), device=dev, generator=g)
        u[0] = 0; u[-1] = 0; u[:, 0] = 0; u[:, -1] = 0
        v = torch.empty_like(u)
        ws = kernels.jacobi_workspace(dev)
        res = torch.zeros(SWEEPS // RES_EVERY, dtype=torch.float64, device=dev)

        def step():
            kernels.jacobi2d(u, v, SWEEPS, RES_EVERY, ws=ws, res=res, check=False)

        def finish():
            kernels.workspace_status(ws)
    else:
        job = slab.SlabJacobi2D(rows_per_rank=rows, cols=GRID, seed=4, res_every=RES_EVERY)

        def step():
            job.run(SWEEPS, check=False)

        def finish():
            job.check()

    clk = ClockSampler(local)
    ms_step, ms_kernel = timed_steps(step, args.steps, args.warmup, world, dist, torch, finish, region=clk)
    updates = rows * GRID * SWEEPS * world
    value = updates / (ms_step * 1e-3) / 1e9

    # ---- e2e through the host-buffer C entries -----------------------------------
    # The headline: `steps` independent pinned host grids through the batch entry
    # (every grid's upload and download inside the timed region; the copies of
    # one grid overlap the sweeps of its neighbours).  Beside it, one grid through
    # the synchronous single-grid entry, whose copies cannot overlap anything.
    e2e = None
    if world == 1:
        host = importlib.import_module("spmd-dialect_b200.host")
        nb = max(2, min(args.steps, 3))
        hbufs = [torch.empty((rows, GRID), dtype=torch.float32, pin_memory=True) for _ in range(nb)]
        grids = [h.numpy() for h in hbufs]
        host.jacobi2d_host_batch(grids, 0, 0)  # warm-up: device slots allocated once, copies only
        for h in hbufs:
            h.copy_(u, non_blocking=False)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        host.jacobi2d_host_batch(grids, SWEEPS, RES_EVERY)
        batch_s = time.perf_counter() - t0
        hbufs[0].copy_(u, non_blocking=False)
        host.jacobi2d_host(grids[0], 2, 0)  # warm-up of the single-grid entry's staging
        hbufs[0].copy_(u, non_blocking=False)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        host.jacobi2d_host(grids[0], SWEEPS, RES_EVERY)
        single_s = time.perf_counter() - t0
        e2e = {"value": round(nb * rows * GRID * SWEEPS / batch_s / 1e9, 3), "unit": "Gcell-updates/s",
               "h2d_bytes_per_step": rows * GRID * 4,
               "d2h_bytes_per_step": rows * GRID * 4 + (SWEEPS // RES_EVERY) * 8,
               "entry": f"spmdb200_jacobi2d_host_batch, {nb} pinned host grids (one per step), wall clock",
               "single_grid": {"value": round(rows * GRID * SWEEPS / single_s / 1e9, 3),
                               "entry": "spmdb200_jacobi2d_host (one pinned grid, copies not overlapped)"}}
        del hbufs, grids
        getattr(importlib.import_module("spmd-dialect_b200._lib"), "lib")().spmdb200_release_cache()
    else:
        e2e = slab.e2e_measure(job, SWEEPS)

    # ---- roofline of the dominant kernel (the persistent sweep kernel) --------------
    plan = sweep_passes(SWEEPS, RES_EVERY)
    alg_bytes = rows * GRID * SWEEPS * bytes_per_update(SWEEPS, RES_EVERY)
    achieved = alg_bytes / (ms_kernel * 1e-3) / 1e9
    kname = "jacobi2d_wave_kernel<%d>" % max(plan, key=lambda f: plan[f] * f)
    ratio = TRAFFIC_OVER_ALGORITHMIC.get(kname)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4),
                "traffic": (round(ratio * alg_bytes) if ratio else None),
                "traffic_basis": "ncu DRAM read+write bytes over algorithmic bytes on a 16384^2 grid in eight-sweep "
                                 "passes (1.077) x the launch's algorithmic bytes",
                "kernel": kname, "peak_kind": f"{peak_kind} hbm_gbs (copy bandwidth)",
                "passes_per_step": {f"{f}_sweep": n for f, n in plan.items() if n},
                "algorithmic_bytes_per_update": round(bytes_per_update(SWEEPS, RES_EVERY), 4),
                "algorithmic_bytes_per_launch": round(alg_bytes),
                # The same time against one-sweep-per-pass traffic (read u, write v: 8 B per update),
                # i.e. how far past the ceiling of any kernel without temporal blocking it runs.
                "single_sweep_bytes_per_update": 8,
                "frac_vs_single_sweep_ceiling": round(rows * GRID * SWEEPS * 8 / (ms_kernel * 1e-3) / 1e9
                                                      / hbm_peak, 4)}

    secondary = None
    multi = None
    if world == 1:
        secondary = secondary_benchmarks(kernels, torch, hbm_peak)
    else:
        job.close()
        multi, multi_ok = multi_gpu_records(slab, shard, kernels, torch, dist, rank, world, args, hbm_peak)
        parity["sharded_sums"] = {"ok": multi_ok}
        parity_ok = parity_ok and multi_ok
    clocks = clk.summary()
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "Gcell-updates/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: torch Philox uniform [0,1) seeded 4 on device, zero boundary; parity cases "
                    "numpy RandomState",
            "config": {"workload": "jacobi2d 5-point, 32768x32768 f32 row slab per GPU, 1000 sweeps, "
                                   "residual every 10 (multi-GPU Jacobi-2D config, weak-scaled)",
                       "grid_per_gpu": [rows, GRID], "global_grid": [rows * world, GRID], "sweeps": SWEEPS,
                       "res_every": RES_EVERY, "parallelism": f"row-slab x{world}",
                       "l2": "inputs (4 GiB per grid) larger than L2; no flush needed"},
            "parity": {**parity, "all_ok": parity_ok},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": args.steps * sum(1 for n in plan.values() if n),
            "clocks": clocks, "secondary": secondary,
        }
        if multi:
            line.update(multi)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not parity_ok:
        print("PARITY FAILURE: a checked result differs from the oracle", file=sys.stderr, flush=True)
        sys.exit(3)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["spmd", "reference"], default="spmd")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_spmd_arm(args)


if __name__ == "__main__":
    main()
