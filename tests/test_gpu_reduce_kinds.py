"""Every spmd.reduce kind on the B200 vs the oracle's serial SCF-order reduce
(oracle_reduce_f32 / oracle_reduce_i32, which restate ReduceToSCFForGPU and its
combine table, lib/Conversion/SPMDToGPU/SPMDToGPU.cpp:425-449).

i32 add/mul/max/min/and/or/xor and f32 max/min are order-independent, so they
must match bit for bit; f32 add and mul (f64 accumulation, one rounding) are
held to 1e-6 of the f64 sum / product (values near 1 keep the product finite).
The serial f32 product chain itself drifts ~sqrt(N) ulps, so it is only a
loose cross-check."""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SIZES = [1, 7, 256, 1000, 65537, 1 << 20]


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("kind", ["add", "mul", "max", "min", "and", "or", "xor"])
@pytest.mark.parametrize("n", SIZES)
def test_i32_kinds_exact(kernels, oracle_mod, kind, n):
    rng = np.random.RandomState(7)
    if kind == "mul":
        a = rng.choice(np.array([1, 1, 1, -1, 3, 5, 7, 2**31 - 1], dtype=np.int32), n).astype(np.int32)
    else:
        a = rng.randint(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
    init = int(rng.randint(-1000, 1000))
    got = int(kernels.reduce(kind, _t(a), init).item())
    assert got == oracle_mod.reduce_i32(kind, a, init), f"i32 {kind} n={n}"


@pytest.mark.parametrize("kind", ["max", "min"])
@pytest.mark.parametrize("n", SIZES)
def test_f32_maxmin_exact(kernels, oracle_mod, kind, n):
    a = (np.random.RandomState(3).random_sample(n) * 200 - 100).astype(np.float32)
    got = np.float32(kernels.reduce(kind, _t(a), 0.5).item())
    want = oracle_mod.reduce_f32(kind, a, 0.5)
    assert got.view(np.uint32) == want.view(np.uint32)


def test_f32_maxmin_nan_and_signed_zero(kernels, oracle_mod):
    base = np.zeros(5000, np.float32)
    base[17] = -0.0
    for kind in ("max", "min"):
        # +0 / -0 ordering (arith.maximumf / minimumf)
        a = base.copy()
        a[::2] = -0.0
        got = np.float32(kernels.reduce(kind, _t(a), -0.0 if kind == "max" else 0.0).item())
        want = oracle_mod.reduce_f32(kind, a, -0.0 if kind == "max" else 0.0)
        assert got.view(np.uint32) == want.view(np.uint32), kind
        # any NaN makes the result NaN
        a = np.random.RandomState(1).random_sample(5000).astype(np.float32)
        a[4321] = np.nan
        assert math.isnan(kernels.reduce(kind, _t(a), 0.0).item())
        assert math.isnan(float(oracle_mod.reduce_f32(kind, a, 0.0)))


@pytest.mark.parametrize("n", SIZES)
def test_f32_add_and_mul(kernels, oracle_mod, n):
    rng = np.random.RandomState(5)
    a = rng.random_sample(n).astype(np.float32)
    got = float(kernels.reduce("add", _t(a), 1.5).item())
    want = 1.5 + float(np.sum(a.astype(np.float64)))
    assert abs(got - want) <= 1e-6 * abs(want)
    m = (1.0 + (rng.random_sample(n) - 0.5) * 1e-3).astype(np.float32)
    got = float(kernels.reduce("mul", _t(m), 2.0).item())
    want = 2.0 * float(np.prod(m.astype(np.float64)))
    assert abs(got - want) <= 1e-6 * abs(want)
    serial = float(oracle_mod.reduce_f32("mul", m, 2.0))
    assert abs(got - serial) <= 1e-3 * abs(serial)


def test_kind_rejected(kernels):
    import torch
    spmd = __import__("importlib").import_module("spmd-dialect_b200._lib")
    with pytest.raises(spmd.SpmdError):
        kernels.reduce("and", torch.ones(4, device="cuda"), 0.0)  # bitwise kinds are integer-only


@pytest.mark.parametrize("kind", ["add", "max", "min", "xor", "mul"])
def test_kinds_staged_and_grid_stride_paths(kernels, oracle_mod, kind):
    """Unit-stride, 16-byte aligned input runs the shared-memory-staged kernel;
    a misaligned or strided view runs the grid-stride one.  Both agree with
    the oracle: bit for bit where the kind is order-independent, within
    1e-6 of the f64 result for f32 add.  The large size spans every SM with a
    ragged tail (n % 4 == 3); n = 0 returns the initial value."""
    import torch
    n = (1 << 24) + 3
    i32 = kind in ("xor", "mul")
    rng = np.random.RandomState(11)
    if kind == "mul":
        a = rng.choice(np.array([1, 1, 1, -1, 3, 2**31 - 1], dtype=np.int32), n).astype(np.int32)
    elif i32:
        a = rng.randint(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
    else:
        a = (rng.random_sample(n) * 200 - 100).astype(np.float32)
    t = _t(a)
    init = 7 if i32 else 0.5
    for view, host in ((t, a), (t[1:], a[1:]), (t[::3], a[::3])):
        got = kernels.reduce(kind, view, init).item()
        if i32:
            assert int(got) == oracle_mod.reduce_i32(kind, np.ascontiguousarray(host), init), kind
        elif kind == "add":
            want = init + float(np.sum(host.astype(np.float64)))
            assert abs(got - want) <= 1e-6 * abs(want)
        else:
            want = oracle_mod.reduce_f32(kind, np.ascontiguousarray(host), init)
            assert np.float32(got).view(np.uint32) == want.view(np.uint32), kind
    empty = torch.empty(0, dtype=t.dtype, device="cuda")
    assert kernels.reduce(kind, empty, init).item() == init
