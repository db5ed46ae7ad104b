"""Generates the golden fixtures in tests/golden/ (run where the reference tree
is available; the fixtures are committed, the tests never read the reference).

    python tests/golden/make_golden.py --reference <reference checkout>
    (or SPMD_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py)

What it pins, and against what:
  * The reference's own numpy references, imported from its harness modules
    (harness/run_ewise.py, harness/run_promoted_stencil.py::cpu_reference,
    harness/run_reduction.py) with a stub standing in for cuda_driver so no
    GPU is touched, on the reference's seeds and sizes
    (RandomState(42) ewise, RandomState(0) stencil and reduction,
    RandomState(99) negative test).
  * The reference's own host harness harness/run_host.py, run unchanged
    against the oracle library (same exported names and ABI as the SCF/OpenMP
    .so files it normally loads); its PASS/FAIL results are recorded in
    reference_harness_run.json.
  * Jacobi-2D/3D and axpy have no reference kernel.  Their fixtures come from an
    independent numpy restatement (vectorised, f32, MLIR source order) so the C
    oracle is cross-checked by a second implementation.
Large-N reduction inputs are not stored: the tests regenerate them from the
seed (numpy's legacy RandomState stream is frozen) and check a SHA-256 of the
bytes stored here.
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import importlib.util
import io
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle import oracle  # noqa: E402

HIER_SIZES = [1, 32, 33, 255, 256, 257, 1000, 1024, 65536, 65537, 1048576, 16777216]


def _load_ref_module(harness: Path, name: str):
    if "cuda_driver" not in sys.modules:
        stub = types.ModuleType("cuda_driver")  # no GPU here: only names used in annotations
        stub.DevicePtr = object
        sys.modules["cuda_driver"] = stub
    spec = importlib.util.spec_from_file_location(f"ref_{name}", harness / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---- independent numpy restatements (no reference kernel exists) -------------------
def np_jacobi2d(U0: np.ndarray, sweeps: int, res_every: int):
    u = U0.astype(np.float32).copy()
    res = []
    k = np.float32(0.2)
    for s in range(1, sweeps + 1):
        v = u.copy()
        if u.shape[0] >= 3 and u.shape[1] >= 3:
            c, n, so = u[1:-1, 1:-1], u[:-2, 1:-1], u[2:, 1:-1]
            e, w = u[1:-1, 2:], u[1:-1, :-2]
            v[1:-1, 1:-1] = ((((c + n) + so) + e) + w) * k
        if res_every and s % res_every == 0:
            d = v.astype(np.float64) - u.astype(np.float64)
            res.append(float(np.sum(d * d)))
        u = v
    return u, np.array(res, dtype=np.float64)


def np_jacobi3d(U0: np.ndarray, sweeps: int, res_every: int):
    u = U0.astype(np.float32).copy()
    res = []
    k = np.float32(1.0) / np.float32(7.0)
    for s in range(1, sweeps + 1):
        v = u.copy()
        if min(u.shape) >= 3:
            c = u[1:-1, 1:-1, 1:-1]
            t = c + u[1:-1, 1:-1, :-2]
            t = t + u[1:-1, 1:-1, 2:]
            t = t + u[1:-1, :-2, 1:-1]
            t = t + u[1:-1, 2:, 1:-1]
            t = t + u[:-2, 1:-1, 1:-1]
            t = t + u[2:, 1:-1, 1:-1]
            v[1:-1, 1:-1, 1:-1] = t * k
        if res_every and s % res_every == 0:
            d = v.astype(np.float64) - u.astype(np.float64)
            res.append(float(np.sum(d * d)))
        u = v
    return u, np.array(res, dtype=np.float64)


def jacobi_init(shape, seed: int) -> np.ndarray:
    """Interior uniform [0,1) from RandomState(seed), boundary 0 (the J2/J3/M2 configs)."""
    rng = np.random.RandomState(seed)
    u = rng.random_sample(shape).astype(np.float32)
    if u.ndim == 2:
        u[0, :] = 0; u[-1, :] = 0; u[:, 0] = 0; u[:, -1] = 0
    else:
        u[0] = 0; u[-1] = 0; u[:, 0] = 0; u[:, -1] = 0; u[:, :, 0] = 0; u[:, :, -1] = 0
    return u


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPMD_REFERENCE_DIR"),
                    help="reference checkout (default: $SPMD_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("give --reference or set SPMD_REFERENCE_DIR")
    harness = Path(args.reference) / "harness"
    if not harness.exists():
        raise SystemExit(f"reference harness not found at {harness}")
    run_ewise = _load_ref_module(harness, "run_ewise")
    run_stencil = _load_ref_module(harness, "run_promoted_stencil")
    run_reduction = _load_ref_module(harness, "run_reduction")
    run_host = _load_ref_module(harness, "run_host")
    meta: dict = {"generator": "tests/golden/make_golden.py", "oracle_threads": oracle.num_threads()}

    # 1. ewise: run_ewise.py test_correctness input stream (RandomState(42), sizes).
    sizes = [32, 100, 1024, 10000]
    rng = np.random.RandomState(42)
    ew = {}
    for n in sizes:
        A = rng.random_sample(n).astype(np.float32)
        B = rng.random_sample(n).astype(np.float32)
        ew[f"A_{n}"], ew[f"B_{n}"], ew[f"C_{n}"] = A, B, A + B  # run_ewise.py:83 reference formula
    np.savez_compressed(HERE / "ewise.npz", sizes=np.array(sizes), **ew)

    # 2. promoted stencil: run_promoted_stencil.py test_correctness (RandomState(0),
    #    A drawn (N+1)x(M+1) and sliced), the reference's cpu_reference on A.
    shapes = [(64, 64), (33, 17), (128, 128), (8, 40)]
    rng = np.random.RandomState(0)
    st = {}
    for (n, m) in shapes:
        A_big = rng.random_sample((n + 1, m + 1)).astype(np.float32)
        A = A_big[:n, :m]
        st[f"Abig_{n}x{m}"] = A_big
        st[f"Bint_{n}x{m}"] = run_stencil.cpu_reference(A)  # interior defined by the reference
        full = np.zeros((n, m), np.float32)
        full[:, :] = (A_big[:n, :m] + A_big[:n, 1:m + 1]) + A_big[1:n + 1, :m]
        st[f"Bfull_{n}x{m}"] = full  # stencil_cpu on the (N+1)x(M+1) host layout
    np.savez_compressed(HERE / "stencil3.npz", shapes=np.array(shapes), **st)

    # 3. reductions: run_reduction.py hierarchical suite (RandomState(0) over HIER_SIZES).
    rng = np.random.RandomState(0)
    red = {"sizes": HIER_SIZES, "np_sum": [], "f64_sum": [], "sha256": []}
    for n in HIER_SIZES:
        A = rng.random_sample(n).astype(np.float32)
        red["np_sum"].append(float(np.sum(A)))  # the reference's yardstick (run_reduction.py:182)
        red["f64_sum"].append(float(np.sum(A.astype(np.float64))))
        red["sha256"].append(sha(A))
    A = rng.random_sample(65536).astype(np.float32)  # the 3x multi-launch array that follows
    red["multi_f64_sum"] = float(np.sum(A.astype(np.float64)))
    red["multi_sha256"] = sha(A)
    A = np.random.RandomState(99).random_sample(1024).astype(np.float32)  # negative test input
    red["negative_f64_sum"] = float(np.sum(A.astype(np.float64)))
    # int32 sum config: N=2^24, values in [0,100) from seed 0.
    Ai = np.random.RandomState(0).randint(0, 100, 1 << 24, dtype=np.int32)
    red["i32_n"] = 1 << 24
    red["i32_sum"] = int(np.sum(Ai.astype(np.int64)))
    red["i32_sha256"] = sha(Ai)
    # f32 sum config: N=2^24, [0,1) from seed 0 (first draw of a fresh RandomState(0)).
    Af = np.random.RandomState(0).random_sample(1 << 24).astype(np.float32)
    red["f32_cfg_f64_sum"] = float(np.sum(Af.astype(np.float64)))
    red["f32_cfg_sha256"] = sha(Af)
    (HERE / "reduction.json").write_text(json.dumps(red, indent=1))

    # 4. axpy (no reference kernel): seed 1, [-1,1), a = 2.5.
    rng = np.random.RandomState(1)
    x = (rng.random_sample(1000) * 2 - 1).astype(np.float32)
    y = (rng.random_sample(1000) * 2 - 1).astype(np.float32)
    np.savez_compressed(HERE / "axpy.npz", x=x, y=y, out=np.float32(2.5) * x + y)

    # 5. Jacobi-2D / 3D (no reference kernel): numpy restatement.
    j2 = {}
    for (h, w, sw, re, seed) in [(34, 70, 7, 2, 2), (5, 9, 3, 1, 2), (130, 260, 4, 1, 4), (3, 3, 2, 1, 2),
                                 (40, 136, 5, 5, 2)]:
        U0 = jacobi_init((h, w), seed)
        fin, res = np_jacobi2d(U0, sw, re)
        key = f"{h}x{w}_s{sw}_r{re}"
        j2[f"U0_{key}"], j2[f"fin_{key}"], j2[f"res_{key}"] = U0, fin, res
    np.savez_compressed(HERE / "jacobi2d.npz", **j2)
    j3 = {}
    for (d, h, w, sw, re, seed) in [(10, 12, 20, 3, 1, 3), (6, 7, 9, 2, 2, 3), (3, 4, 5, 1, 1, 3)]:
        U0 = jacobi_init((d, h, w), seed)
        fin, res = np_jacobi3d(U0, sw, re)
        key = f"{d}x{h}x{w}_s{sw}_r{re}"
        j3[f"U0_{key}"], j3[f"fin_{key}"], j3[f"res_{key}"] = U0, fin, res
    np.savez_compressed(HERE / "jacobi3d.npz", **j3)

    # 6. The reference's host harness, unchanged, driving the oracle library.
    so = str(oracle.lib_path())
    runs = {}
    for label, fn, arg in [
        ("run_ewise", run_host.run_ewise, [32, 100, 1024, 1000000]),
        ("run_stencil", run_host.run_stencil, [(64, 64), (128, 128), (511, 513)]),
        ("run_reduction", run_host.run_reduction, [1024, 65536, 1048576]),
        ("run_reduction_hierarchical", run_host.run_reduction_hierarchical, [1, 255, 257, 65537, 1048576]),
    ]:
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            ok = bool(fn(so, arg))
        runs[label] = {"args": [list(a) if isinstance(a, tuple) else a for a in arg], "pass": ok,
                       "stdout": buf.getvalue().splitlines()}
        if not ok:
            raise SystemExit(f"reference harness {label} FAILED on the oracle:\n{buf.getvalue()}")
    meta["reference_harness_run"] = runs
    meta["reference_numpy_refs"] = ["harness/run_ewise.py:83", "harness/run_promoted_stencil.py:111-116",
                                    "harness/run_reduction.py:182"]
    (HERE / "reference_harness_run.json").write_text(json.dumps(meta, indent=1))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
