"""Drop-in checks at the reference's two boundaries, on the B200.

1. spmdb200_kernels.cubin loaded through a driver-API client with the
   reference harness's surface, kernels fetched BY THE REFERENCE'S NAMES and
   launched with the reference's exact parameter lists and launch shapes
   (harness/run_ewise.py:53-70, run_promoted_stencil.py:68-108,
   run_reduction.py:46-134), checked with the reference's tolerances and, where
   the arithmetic is order-pinned, bit-exactly against the oracle.
2. The reference-named host entries of libspmdb200.so called exactly the way
   harness/run_host.py calls the SCF/OpenMP libraries (numpy buffers, unpacked
   descriptors), computing on the GPU."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import assert_bits_equal, spmd_mod

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cd():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    drv = spmd_mod("cuda_driver")
    drv.init()
    return drv


@pytest.fixture(scope="module")
def module(cd):
    return cd.load_cubin(str(spmd_mod("_lib").CUBIN_PATH))


def memref1d(ptr, n):
    return (ptr, ptr, 0, n, 1)


@pytest.mark.parametrize("tile", [32, 256])
def test_ewise_kernel_reference_launch(cd, module, oracle_mod, tile):
    fn = cd.get_function(module, "ewise_kernel")
    rng = np.random.RandomState(42)
    for n in [32, 100, 1024, 10000, 1000000, 33, 1]:
        a = rng.random_sample(n).astype(np.float32)
        b = rng.random_sample(n).astype(np.float32)
        ad, bd, cdv = cd.alloc(a.nbytes), cd.alloc(b.nbytes), cd.alloc(a.nbytes)
        cd.memcpy_h2d(ad, a)
        cd.memcpy_h2d(bd, b)
        cd.launch(fn, (math.ceil(n / tile), 1, 1), (tile, 1, 1), tile, n,
                  *memref1d(ad, n), *memref1d(bd, n), *memref1d(cdv, n))
        cd.synchronize()
        c = np.empty(n, np.float32)
        cd.memcpy_d2h(c, cdv)
        for p in (ad, bd, cdv):
            p.free()
        assert float(np.max(np.abs(c - (a + b)))) < 1e-5  # run_ewise.py:97-99
        assert_bits_equal(c, oracle_mod.ewise(a, b), f"ewise_kernel n={n}")


@pytest.mark.parametrize("tr,tc", [(32, 8), (64, 8), (16, 16)])
def test_promoted_stencil_kernel_reference_launch(cd, module, oracle_mod, tr, tc):
    square = tr == tc
    fn = cd.get_function(module, "promoted_stencil_kernel_square" if square else "promoted_stencil_kernel")
    rng = np.random.RandomState(0)
    for (n, m) in [(64, 64), (128, 128), (512, 512), (1024, 1024)]:
        a_big = rng.random_sample((n + 1, m + 1)).astype(np.float32)
        a = np.ascontiguousarray(a_big[:n, :m])
        ad, bd = cd.alloc(a.nbytes), cd.alloc(a.nbytes)
        cd.memcpy_h2d(ad, a)
        grid = (math.ceil(n / tr), math.ceil(m / tc), 1)
        block = ((tr + 1) * (tc + 1), 1, 1)
        desc_a = (ad, ad, 0, n, m, m, 1)
        desc_b = (bd, bd, 0, n, m, m, 1)
        if square:
            cd.launch(fn, grid, block, tr, *desc_a, 1, *desc_b)
        else:
            cd.launch(fn, grid, block, tr, tc, *desc_a, 1, *desc_b)
        cd.synchronize()
        b = np.zeros((n, m), np.float32)
        cd.memcpy_d2h(b, bd)
        ad.free()
        bd.free()
        ref = np.zeros_like(a)
        ref[: n - 1, : m - 1] = a[: n - 1, : m - 1] + a[: n - 1, 1:m] + a[1:n, : m - 1]
        interior = (slice(0, n - 1), slice(0, m - 1))
        assert float(np.max(np.abs(b[interior] - ref[interior]))) < 1e-4  # run_promoted_stencil.py:139-141
        assert_bits_equal(b, oracle_mod.stencil3(a, n, m), f"promoted {n}x{m} tile {tr}x{tc}")


def _hier(cd, fn, a, tile, out_init=True, out=None):
    n = a.size
    ad = cd.alloc(max(a.nbytes, 4))
    cd.memcpy_h2d(ad, a)
    od = out or cd.alloc(4)
    if out_init:
        cd.memset(od, 0, 4)
    cd.launch(fn, (max(math.ceil(n / tile), 1), 1, 1), (tile, 1, 1), tile, n, ad, od)
    cd.synchronize()
    r = np.zeros(1, np.float32)
    cd.memcpy_d2h(r, od)
    ad.free()
    return float(r[0]), od


def test_hierarchical_sum_kernel_reference_suite(cd, module, oracle_mod):
    fn = cd.get_function(module, "hierarchical_sum_kernel")
    rng = np.random.RandomState(0)
    for n in [1, 32, 33, 255, 256, 257, 1000, 1024, 65536, 65537, 1048576, 16777216]:
        a = rng.random_sample(n).astype(np.float32)
        got, od = _hier(cd, fn, a, 256)
        od.free()
        ref = float(np.sum(a))
        assert abs(got - ref) / max(abs(ref), 1e-6) < 1e-3  # run_reduction.py:137-141
        f64 = oracle_mod.sum_f64(a)
        assert abs(got - f64) / f64 < 1e-5
    for n in (256, 1024):
        got, od = _hier(cd, fn, np.zeros(n, np.float32), 256)
        od.free()
        assert got == 0.0
        got, od = _hier(cd, fn, np.ones(n, np.float32), 256)
        od.free()
        assert got == float(n)
    # negative self-test: second launch without re-zeroing must FAIL the check
    a = np.random.RandomState(99).random_sample(1024).astype(np.float32)
    _, od = _hier(cd, fn, a, 256)
    got, od = _hier(cd, fn, a, 256, out_init=False, out=od)
    od.free()
    ref = float(np.sum(a))
    assert abs(got - ref) / ref >= 1e-3


def test_atomic_sum_kernel_reference_launch(cd, module):
    fn = cd.get_function(module, "atomic_sum_kernel")
    rng = np.random.RandomState(0)
    for n in [1024, 65536, 1048576]:
        a = rng.random_sample(n).astype(np.float32)
        ad, od = cd.alloc(a.nbytes), cd.alloc(4)
        cd.memcpy_h2d(ad, a)
        cd.memset(od, 0, 4)
        cd.launch(fn, (math.ceil(n / 256), 1, 1), (256, 1, 1), 256, n, ad, ad, 0, n, 1, od, od, 0)
        cd.synchronize()
        r = np.zeros(1, np.float32)
        cd.memcpy_d2h(r, od)
        ad.free()
        od.free()
        ref = float(np.sum(a))
        assert abs(float(r[0]) - ref) / ref < 1e-3


# ---------------------------------------------------------------- run_host.py-style
def test_run_host_ewise(host_api, oracle_mod):
    rng = np.random.RandomState(42)
    for n in [32, 100, 1024, 1000000]:
        a = rng.random_sample(n).astype(np.float32)
        b = rng.random_sample(n).astype(np.float32)
        c = np.zeros(n, np.float32)
        host_api.ewise(a, b, c, n)
        assert float(np.max(np.abs(c - (a + b)))) < 1e-5
        assert_bits_equal(c, oracle_mod.ewise(a, b))


def test_run_host_stencil(host_api, oracle_mod):
    rng = np.random.RandomState(0)
    for (n, m) in [(64, 64), (128, 128), (511, 513)]:
        a = rng.random_sample((n + 1, m + 1)).astype(np.float32)
        b = np.zeros((n, m), np.float32)
        host_api.stencil_cpu(a, b, n, m)
        assert_bits_equal(b, oracle_mod.stencil3(a, n, m), f"stencil_cpu {n}x{m}")


@pytest.mark.parametrize("name", ["atomic_sum", "hierarchical_sum"])
def test_run_host_reductions(host_api, oracle_mod, name):
    rng = np.random.RandomState(0)
    for n in [1, 255, 257, 65537, 1048576]:
        a = rng.random_sample(n).astype(np.float32)
        out = np.zeros(1, np.float32)
        getattr(host_api, name)(a, out, n)
        f64 = oracle_mod.sum_f64(a)
        assert abs(float(out[0]) - f64) / f64 <= 1e-6


def test_run_host_strided_views(host_api, oracle_mod):
    rng = np.random.RandomState(3)
    big = rng.random_sample(3000).astype(np.float32)
    a, b = big[::3], big[1::3]
    c = np.zeros(2000, np.float32)[::2]
    host_api.ewise(a, b, c)
    assert_bits_equal(c, oracle_mod.ewise(np.ascontiguousarray(a), np.ascontiguousarray(b)))


def test_e2e_host_entries(host_api, oracle_mod):
    rng = np.random.RandomState(1)
    x = (rng.random_sample(100003) * 2 - 1).astype(np.float32)
    y = (rng.random_sample(100003) * 2 - 1).astype(np.float32)
    want = oracle_mod.axpy(2.5, x, y)
    host_api.axpy_host(2.5, x, y)
    assert_bits_equal(y, want, "axpy_host")
    ai = np.random.RandomState(0).randint(0, 100, 1 << 20, dtype=np.int32)
    o = np.zeros(1, np.int32)
    host_api.sum_i32_host(ai, o)
    assert int(o[0]) == oracle_mod.sum_i32(ai)
    af = np.random.RandomState(0).random_sample(1 << 20).astype(np.float32)
    of = np.zeros(1, np.float32)
    host_api.sum_f32_host(af, of)
    assert abs(float(of[0]) - oracle_mod.sum_f64(af)) / oracle_mod.sum_f64(af) <= 1e-6


def test_invalid_descriptor_raises_on_gpu(host_api):
    lib_mod = spmd_mod("_lib")
    a = np.ones(10, np.float32)
    with pytest.raises(lib_mod.SpmdError):
        host_api.ewise(a, a, np.zeros(10, np.float32), 20)  # loop bound > sizes
