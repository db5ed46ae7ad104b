"""spmd.kernel functions run through the textual-MLIR shim on the GPU, called
with their own argument lists, against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ROOT, assert_bits_equal, spmd_mod

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fns(kernels):
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


def test_top_level_reduces_and_float_identities(kernels, oracle_mod):
    """A returned top-level spmd.reduce, one stored to out[c], and a max
    reduction whose init is a hexadecimal -inf, through their bindings."""
    from test_mlir_shim import _FORMS
    shim = spmd_mod("mlir_shim")
    fns = shim.load(_FORMS, skip_unmapped=True)
    x = _r(300001, 21)
    tx = torch.from_numpy(x).cuda()
    got = fns["sum_returned"](tx, 300001)
    exact = oracle_mod.sum_f64(x)
    assert isinstance(got, float) and abs(got - exact) <= 1e-6 * abs(exact)
    o = torch.tensor(-7.0, device="cuda")
    fns["max_f32"](tx, o, 300001)
    assert float(o.item()) == float(x.max())
    stored = shim.load("""
func.func @sum_stored(%A: memref<?xf32>, %out: memref<3xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c2 = arith.constant 2 : index
  %z = arith.constant 0.0 : f32
  %s = "spmd.reduce"(%c0, %N, %c1, %z) ({
  ^bb0(%k: index):
    %v = memref.load %A[%k] : memref<?xf32>
    "spmd.yield"(%v) : (f32) -> ()
  }) {"spmd.kind" = #spmd.reduction_kind<add>} : (index, index, index, f32) -> f32
  memref.store %s, %out[%c2] : memref<3xf32>
  func.return
}
""")
    out = torch.full((3,), 5.0, device="cuda")
    stored["sum_stored"](tx, out, 1000)
    got = out.cpu().numpy()
    assert got[0] == 5.0 and got[1] == 5.0
    assert abs(float(got[2]) - oracle_mod.sum_f64(x[:1000])) <= 1e-6 * oracle_mod.sum_f64(x[:1000])


def test_guarded_stores(fns):
    rs = np.random.RandomState(33)
    a = rs.uniform(-2, 2, 5001).astype(np.float32)
    ta = torch.from_numpy(a).cuda()
    fns["clamp_guarded"](ta, 5000, 0.5)
    want = a.copy()
    want[:5000] = np.where(a[:5000] > np.float32(0.5), np.float32(0.5), a[:5000])
    assert np.array_equal(ta.cpu().numpy(), want)
    m = rs.uniform(-2, 2, (33, 70)).astype(np.float32)
    tb = torch.zeros((33, 70), device="cuda")
    fns["abs_if_else"](torch.from_numpy(m).cuda(), tb, 33, 70)
    assert np.array_equal(tb.cpu().numpy(), np.where(m >= 0, m, -m).astype(np.float32))


def test_spmd_if_value(fns):
    rs = np.random.RandomState(35)
    a, b = rs.randn(3001).astype(np.float32), rs.randn(3001).astype(np.float32)
    tc = torch.zeros(3001, device="cuda")
    fns["select_by_if"](torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), tc, 3001)
    assert np.array_equal(tc.cpu().numpy(), np.where(a < b, b - a, a - b).astype(np.float32))


def test_nonlinear_stencils(fns):
    rs = np.random.RandomState(38)
    a = rs.randn(4000).astype(np.float32)
    tb = torch.full((4000,), 9.0, device="cuda")
    fns["max_filter_interior"](torch.from_numpy(a).cuda(), tb, 3999)
    want = np.full(4000, 9.0, np.float32)
    want[1:3999] = np.maximum(a[:3998], a[2:]) - a[1:3999]
    assert np.array_equal(tb.cpu().numpy(), want)
    m = rs.randn(70, 130).astype(np.float32)
    tu = torch.zeros((70, 130), device="cuda")
    fns["upwind2d"](torch.from_numpy(m).cuda(), tu, 69, 130)
    c = m[1:69]
    got = tu.cpu().numpy()
    assert np.array_equal(got[1:69], np.where(c > 0, c - m[:68], m[2:] - c).astype(np.float32))
    assert not got[0].any() and not got[69].any()
    shim = spmd_mod("mlir_shim")
    with pytest.raises(shim.ShimError):  # a shifted view would start before the memref
        fns["max_filter_interior"](torch.from_numpy(a).cuda(), tb, 4001)
