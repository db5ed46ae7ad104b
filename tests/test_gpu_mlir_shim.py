"""spmd.kernel functions run through the textual-MLIR shim on the GPU, called
with their own argument lists, against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ROOT, assert_bits_equal, spmd_mod

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fns():
    shim = spmd_mod("mlir_shim")
    return shim.load((ROOT / "tests" / "mlir" / "kernels.mlir").read_text(), skip_unmapped=True)


def _r(shape, seed):
    return np.random.RandomState(seed).random_sample(shape).astype(np.float32)


def test_ewise_and_axpy(fns, oracle_mod):
    a, b = _r(1000, 1), _r(1000, 2)
    ta, tb, tc = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.zeros(1000, device="cuda")
    fns["ewise"](ta, tb, tc, 777)
    got = tc.cpu().numpy()
    assert_bits_equal(got[:777], oracle_mod.ewise(a[:777], b[:777]))
    assert not got[777:].any()
    y = _r(1000, 3)
    ty = torch.from_numpy(y).cuda()
    fns["axpy"](ta, ty, 1000)
    assert_bits_equal(ty.cpu().numpy(), oracle_mod.axpy(2.5, a, y))


def test_promoted_stencil_and_jacobi(fns, oracle_mod):
    a = _r((130, 70), 4)
    tb = torch.zeros((129, 69), device="cuda")
    fns["promoted_stencil"](torch.from_numpy(a).cuda(), tb, 129, 69)
    assert_bits_equal(tb.cpu().numpy(), oracle_mod.stencil3(a, 129, 69))
    u = _r((64, 96), 5)
    tv = torch.zeros((64, 96), device="cuda")
    fns["jacobi_interior"](torch.from_numpy(u).cuda(), tv, 64, 96)
    want = oracle_mod.stencil_nd(u, u.shape, [[0, 0], [-1, 0], [1, 0], [0, 1], [0, -1]], scale=0.2)
    got = tv.cpu().numpy()
    assert_bits_equal(got, want)
    one, _ = oracle_mod.jacobi2d(u, 1, 0)
    assert_bits_equal(got[1:-1, 1:-1], one[1:-1, 1:-1])


def test_stepped_and_lower_bound(fns, oracle_mod):
    a = _r(501, 6)
    tb = torch.zeros(500, device="cuda")
    fns["pairs_stepped"](torch.from_numpy(a).cuda(), tb, 500)
    assert_bits_equal(tb.cpu().numpy(), oracle_mod.stencil_nd(a, (500,), [[0], [1]], steps=[2]))
    tb2 = torch.zeros(501, device="cuda")
    fns["smooth_interior"](torch.from_numpy(a).cuda(), tb2, 500)
    want = np.zeros(501, np.float32)
    want[1:500] = (np.float32(0.5) * a[0:499]) + (np.float32(0.5) * a[2:501])
    assert_bits_equal(tb2.cpu().numpy(), want)


def test_reductions(fns, oracle_mod):
    x = _r(1 << 20, 7)
    out = torch.zeros(1, device="cuda")
    fns["hierarchical_sum"](torch.from_numpy(x).cuda(), out.reshape(()), 1 << 20)
    exact = oracle_mod.sum_f64(x)
    assert abs(float(out.item()) - exact) <= 1e-5 * abs(exact)
    v = np.random.RandomState(8).randint(-10**9, 10**9, size=123457).astype(np.int32)
    o = torch.tensor([-5], dtype=torch.int32, device="cuda")
    fns["max_i32"](torch.from_numpy(v).cuda(), o.reshape(()), 123457)
    assert int(o.item()) == max(int(v.max()), -5)
