"""The CPU oracle against the golden fixtures (tests/golden/, made by
make_golden.py from the reference's own harness code and seeds, plus an
independent numpy restatement for the configurations the reference has no
kernel for).  Bit-exact wherever the reference arithmetic is order-pinned."""
from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN, assert_bits_equal, jacobi_init


def test_reference_harness_passed_on_oracle():
    meta = json.loads((GOLDEN / "reference_harness_run.json").read_text())
    runs = meta["reference_harness_run"]
    assert set(runs) == {"run_ewise", "run_stencil", "run_reduction", "run_reduction_hierarchical"}
    assert all(r["pass"] for r in runs.values())


def test_ewise_golden(oracle_mod):
    z = np.load(GOLDEN / "ewise.npz")
    for n in z["sizes"]:
        assert_bits_equal(oracle_mod.ewise(z[f"A_{n}"], z[f"B_{n}"]), z[f"C_{n}"], f"ewise {n}")


def test_axpy_golden(oracle_mod):
    z = np.load(GOLDEN / "axpy.npz")
    assert_bits_equal(oracle_mod.axpy(2.5, z["x"], z["y"]), z["out"], "axpy")


def test_stencil3_golden(oracle_mod):
    z = np.load(GOLDEN / "stencil3.npz")
    for n, m in z["shapes"]:
        a_big = z[f"Abig_{n}x{m}"]
        # host layout: A is (N+1)x(M+1), every output cell defined
        assert_bits_equal(oracle_mod.stencil3(a_big, n, m), z[f"Bfull_{n}x{m}"], f"stencil_cpu {n}x{m}")
        # device layout: A is N x M; the reference defines the interior only
        a = np.ascontiguousarray(a_big[:n, :m])
        got = oracle_mod.stencil3(a, n, m)
        assert_bits_equal(got[: n - 1, : m - 1], z[f"Bint_{n}x{m}"][: n - 1, : m - 1], f"interior {n}x{m}")


def _regen(n: int, seed_stream) -> np.ndarray:
    return seed_stream.random_sample(n).astype(np.float32)


def test_reduction_golden(oracle_mod):
    red = json.loads((GOLDEN / "reduction.json").read_text())
    rng = np.random.RandomState(0)
    for n, np_sum, f64, digest in zip(red["sizes"], red["np_sum"], red["f64_sum"], red["sha256"]):
        a = _regen(n, rng)
        assert hashlib.sha256(a.tobytes()).hexdigest() == digest, "RandomState stream drifted"
        assert oracle_mod.sum_f64(a) == pytest.approx(f64, rel=1e-12)
        # the reference's own check: rel_err < 1e-3 against np.sum (run_reduction.py:137-141)
        for got in (oracle_mod.hierarchical_sum(a), oracle_mod.atomic_sum(a)):
            assert abs(float(got) - np_sum) / max(abs(np_sum), 1e-6) < 1e-3
    # known answers (run_reduction.py:187-201)
    for n in (256, 1024):
        assert oracle_mod.hierarchical_sum(np.zeros(n, np.float32)) == 0.0
        assert oracle_mod.hierarchical_sum(np.ones(n, np.float32)) == float(n)


def test_int32_sum_golden(oracle_mod):
    red = json.loads((GOLDEN / "reduction.json").read_text())
    a = np.random.RandomState(0).randint(0, 100, red["i32_n"], dtype=np.int32)
    assert hashlib.sha256(a.tobytes()).hexdigest() == red["i32_sha256"]
    assert oracle_mod.sum_i32(a) == red["i32_sum"]


def test_int32_sum_wraps(oracle_mod):
    a = np.array([2**31 - 1, 2**31 - 1, 5, -7], dtype=np.int32)
    want = np.array([int(a.astype(np.int64).sum()) & 0xFFFFFFFF], dtype=np.uint32).view(np.int32)[0]
    assert oracle_mod.sum_i32(a) == int(want)


def test_jacobi2d_golden(oracle_mod):
    z = np.load(GOLDEN / "jacobi2d.npz")
    keys = sorted(k[3:] for k in z.files if k.startswith("U0_"))
    assert keys
    for key in keys:
        sw = int(key.split("_s")[1].split("_")[0])
        re = int(key.split("_r")[1])
        fin, res = oracle_mod.jacobi2d(z[f"U0_{key}"], sw, re)
        assert_bits_equal(fin, z[f"fin_{key}"], f"jacobi2d {key}")
        np.testing.assert_allclose(res, z[f"res_{key}"], rtol=1e-12, atol=0)


def test_jacobi3d_golden(oracle_mod):
    z = np.load(GOLDEN / "jacobi3d.npz")
    keys = sorted(k[3:] for k in z.files if k.startswith("U0_"))
    assert keys
    for key in keys:
        sw = int(key.split("_s")[1].split("_")[0])
        re = int(key.split("_r")[1])
        fin, res = oracle_mod.jacobi3d(z[f"U0_{key}"], sw, re)
        assert_bits_equal(fin, z[f"fin_{key}"], f"jacobi3d {key}")
        np.testing.assert_allclose(res, z[f"res_{key}"], rtol=1e-12, atol=0)


def test_jacobi2d_thread_count_independent(oracle_mod, monkeypatch):
    """Oracle results do not depend on the OpenMP thread count (row-ordered residual)."""
    u0 = jacobi_init((67, 131), 2)
    fin1, res1 = oracle_mod.jacobi2d(u0, 6, 3)
    fin2, res2 = oracle_mod.jacobi2d(u0, 6, 3)
    assert_bits_equal(fin1, fin2)
    assert np.array_equal(res1, res2)


def test_negative_self_test_detects_double_accumulation(oracle_mod):
    """Mirror of run_reduction.py:214-264 on the oracle: accumulating twice
    without re-zeroing must FAIL the 1e-3 check."""
    red = json.loads((GOLDEN / "reduction.json").read_text())
    a = np.random.RandomState(99).random_sample(1024).astype(np.float32)
    once = float(oracle_mod.hierarchical_sum(a))
    twice = float(oracle_mod.hierarchical_sum(a, init=once))
    ref = red["negative_f64_sum"]
    assert abs(once - ref) / ref < 1e-3
    assert abs(twice - ref) / ref >= 1e-3
