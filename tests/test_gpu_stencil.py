"""Promoted stencils on the B200 vs the oracle: bit-exact grids, residuals
within 1e-12 relative (f64 sums in a different order).

Covers the 3-point promoted stencil of the reference (device N x M layout and
the (N+1) x (M+1) host layout), Jacobi-2D on the persistent TMA path
(pitch-aligned) and the per-sweep path (any pitch), Jacobi-3D, ragged and
tiny shapes, odd/even sweep counts, and the 4096^2 x 100 and 512^3 x 50 configs."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, assert_bits_equal, jacobi_init

pytestmark = pytest.mark.gpu

RES_RTOL = 1e-12


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---------------------------------------------------------------- 3-point stencil
@pytest.mark.parametrize("shape", [(64, 64), (128, 128), (511, 513), (1, 1), (33, 9), (17, 300), (1000, 7)])
def test_stencil3_device_layout(kernels, oracle_mod, shape):
    import torch
    n, m = shape
    a = np.random.RandomState(0).random_sample((n, m)).astype(np.float32)
    out = torch.zeros((n, m), device="cuda")
    kernels.stencil3pt(_t(a), out)
    assert_bits_equal(out.cpu().numpy(), oracle_mod.stencil3(a, n, m), f"stencil3 {shape}")


def test_stencil3_golden(kernels):
    import torch
    z = np.load(GOLDEN / "stencil3.npz")
    for n, m in z["shapes"]:
        a_big = z[f"Abig_{n}x{m}"]
        out = torch.zeros((n, m), device="cuda")
        kernels.stencil3pt(_t(a_big), out)  # host-layout semantics: A is (N+1)x(M+1)
        assert_bits_equal(out.cpu().numpy(), z[f"Bfull_{n}x{m}"], f"golden full {n}x{m}")
        out2 = torch.zeros((n, m), device="cuda")
        kernels.stencil3pt(_t(a_big[:n, :m]), out2)  # the reference's device layout
        got = out2.cpu().numpy()[: n - 1, : m - 1]
        assert_bits_equal(got, z[f"Bint_{n}x{m}"][: n - 1, : m - 1], f"golden interior {n}x{m}")


# ---------------------------------------------------------------- Jacobi-2D
def _run_j2(kernels, u0, sweeps, res_every, pitch=None):
    import torch
    h, w = u0.shape
    if pitch is None:
        u = _t(u0)
        v = torch.empty_like(u)
    else:
        ub = torch.zeros((h, pitch), device="cuda")
        vb = torch.zeros((h, pitch), device="cuda")
        ub[:, :w] = _t(u0)
        u, v = ub[:, :w], vb[:, :w]
    fin, res = kernels.jacobi2d(u, v, sweeps, res_every)
    return fin.cpu().numpy(), (res.cpu().numpy() if res is not None else np.zeros(0))


J2_CASES = [
    # (h, w, sweeps, res_every, pitch)  pitch None = dense
    (34, 70, 7, 2, 72),      # TMA path (pitch 72 = 288 B), W not a multiple of 128
    (5, 9, 3, 1, 12),
    (130, 260, 4, 1, None),  # dense 260 -> 1040 B rows: TMA path
    (3, 3, 2, 1, 4),
    (2, 2, 3, 1, 4),
    (1, 5, 2, 1, 8),
    (40, 136, 5, 5, None),
    (257, 129, 6, 3, 132),
    (511, 513, 5, 1, None),  # 2052-byte rows: per-sweep path
    (33, 33, 4, 2, None),    # 132-byte rows: per-sweep path
    (1, 1, 1, 1, 4),
    (64, 1024, 11, 1, None),
    # grids with interior tiles (the unmasked path) for every pass kind:
    # passes no longer than the residual interval, so residual intervals of
    # 1-5 give single-, two- and four-sweep passes, residuals landing in each
    (300, 1000, 7, 3, None),
    (200, 700, 9, 1, 704),
    (260, 1100, 6, 2, None),
    (333, 777, 12, 4, 780),
    (520, 1300, 17, 3, None),
    (130, 245, 16, 5, 248),
    # tiny grids through multi-sweep passes: boxes reach far past every edge
    (5, 9, 8, 1, 12),
    (3, 3, 9, 1, 4),
    (1, 5, 8, 2, 8),
    (2, 130, 16, 4, None),
    (41, 121, 13, 13, 124),
    (2, 130, 24, 8, None),
    (6, 7, 17, 0, 8),
    # eight-sweep passes (residual interval >= 8 or none): interior and edge
    # tiles, the residual on every sweep position of a pass, eight-, four-,
    # two- and single-sweep passes in one run
    (300, 1000, 17, 8, None),
    (520, 1300, 40, 10, None),
    (260, 1100, 16, 0, 1104),
    (700, 2100, 31, 0, None),
    (333, 777, 65, 13, 780),
    (41, 121, 33, 16, 124),
    (1024, 4096, 80, 9, None),
]


@pytest.mark.parametrize("case", J2_CASES, ids=lambda c: f"{c[0]}x{c[1]}_s{c[2]}_p{c[4]}")
def test_jacobi2d_matches_oracle(kernels, oracle_mod, case):
    h, w, sw, re, pitch = case
    u0 = jacobi_init((h, w), 2)
    fin, res = _run_j2(kernels, u0, sw, re, pitch)
    want, wres = oracle_mod.jacobi2d(u0, sw, re)
    assert_bits_equal(fin, want, f"jacobi2d {case}")
    np.testing.assert_allclose(res, wres, rtol=RES_RTOL, atol=1e-300)


def test_jacobi2d_golden(kernels):
    z = np.load(GOLDEN / "jacobi2d.npz")
    for key in sorted(k[3:] for k in z.files if k.startswith("U0_")):
        sw = int(key.split("_s")[1].split("_")[0])
        re = int(key.split("_r")[1])
        fin, res = _run_j2(kernels, z[f"U0_{key}"], sw, re)
        assert_bits_equal(fin, z[f"fin_{key}"], f"golden jacobi2d {key}")
        np.testing.assert_allclose(res, z[f"res_{key}"], rtol=RES_RTOL)


def test_jacobi2d_nonzero_boundary_is_fixed(kernels, oracle_mod):
    u0 = np.random.RandomState(11).random_sample((70, 300)).astype(np.float32)  # boundary not 0
    fin, res = _run_j2(kernels, u0, 9, 3)
    want, wres = oracle_mod.jacobi2d(u0, 9, 3)
    assert_bits_equal(fin, want, "nonzero boundary")
    assert_bits_equal(fin[0], u0[0]) and assert_bits_equal(fin[:, -1], u0[:, -1])
    np.testing.assert_allclose(res, wres, rtol=RES_RTOL)


def test_jacobi2d_config_4096_100_sweeps(kernels, oracle_mod):
    """J2: 4096^2, interior [0,1) seed 2, zero boundary, 100 ping-pong sweeps."""
    u0 = jacobi_init((4096, 4096), 2)
    fin, res = _run_j2(kernels, u0, 100, 10)
    want, wres = oracle_mod.jacobi2d(u0, 100, 10)
    assert_bits_equal(fin, want, "J2 4096^2 x 100")
    np.testing.assert_allclose(res, wres, rtol=RES_RTOL)


def test_jacobi2d_repeat_is_deterministic(kernels):
    u0 = jacobi_init((300, 1000), 2)
    a = _run_j2(kernels, u0, 10, 1)
    b = _run_j2(kernels, u0, 10, 1)
    assert_bits_equal(a[0], b[0])
    assert np.array_equal(a[1], b[1])


def test_jacobi2d_host_entry_e2e(host_api, oracle_mod):
    u0 = jacobi_init((200, 333), 2)
    u = u0.copy()
    _, res = host_api.jacobi2d_host(u, 7, 7)
    want, wres = oracle_mod.jacobi2d(u0, 7, 7)
    assert_bits_equal(u, want, "jacobi2d_host")
    np.testing.assert_allclose(res, wres, rtol=RES_RTOL)


# ---------------------------------------------------------------- Jacobi-3D
def _run_j3(kernels, u0, sweeps, res_every):
    import torch
    u = _t(u0)
    v = torch.empty_like(u)
    fin, res = kernels.jacobi3d(u, v, sweeps, res_every)
    return fin.cpu().numpy(), (res.cpu().numpy() if res is not None else np.zeros(0))


@pytest.mark.parametrize("shape,sw,re", [((10, 12, 20), 3, 1), ((6, 7, 9), 2, 2), ((3, 4, 5), 1, 1),
                                         ((33, 17, 130), 5, 1), ((64, 64, 64), 4, 2), ((2, 2, 2), 2, 1),
                                         # x-contiguous rows of a multiple of 16 bytes: persistent TMA path
                                         ((33, 17, 132), 5, 1), ((5, 3, 4), 3, 1), ((17, 50, 136), 4, 2),
                                         ((40, 33, 260), 7, 7), ((1, 1, 4), 2, 1),
                                         # longer runs on the persistent path: residuals at odd and even
                                         # sweeps, ragged and exact tile shapes
                                         ((37, 45, 300), 9, 2), ((20, 29, 132), 8, 1), ((5, 16, 128), 4, 4),
                                         ((64, 30, 260), 12, 3), ((17, 14, 120), 6, 5), ((33, 3, 8), 5, 1),
                                         ((3, 40, 244), 4, 1)])
def test_jacobi3d_matches_oracle(kernels, oracle_mod, shape, sw, re):
    u0 = jacobi_init(shape, 3)
    fin, res = _run_j3(kernels, u0, sw, re)
    want, wres = oracle_mod.jacobi3d(u0, sw, re)
    assert_bits_equal(fin, want, f"jacobi3d {shape}")
    np.testing.assert_allclose(res, wres, rtol=RES_RTOL, atol=1e-300)


def test_jacobi3d_golden(kernels):
    z = np.load(GOLDEN / "jacobi3d.npz")
    for key in sorted(k[3:] for k in z.files if k.startswith("U0_")):
        sw = int(key.split("_s")[1].split("_")[0])
        re = int(key.split("_r")[1])
        fin, res = _run_j3(kernels, z[f"U0_{key}"], sw, re)
        assert_bits_equal(fin, z[f"fin_{key}"], f"golden jacobi3d {key}")
        np.testing.assert_allclose(res, z[f"res_{key}"], rtol=RES_RTOL)


def test_jacobi3d_config_512_50_sweeps(kernels, oracle_mod):
    """J3: 512^3, interior [0,1) seed 3, zero boundary, 50 sweeps."""
    u0 = jacobi_init((512, 512, 512), 3)
    fin, res = _run_j3(kernels, u0, 50, 10)
    want, wres = oracle_mod.jacobi3d(u0, 50, 10)
    assert_bits_equal(fin, want, "J3 512^3 x 50")
    np.testing.assert_allclose(res, wres, rtol=RES_RTOL)


@pytest.mark.parametrize("pinned", [True, False])
def test_jacobi2d_host_batch_matches_oracle(host_api, oracle_mod, pinned):
    """Five independent grids through the batch host entry (two device slots,
    each reused twice; pinned grids overlap their copies with the sweeps,
    pageable ones do not): every grid and its residuals equal the oracle's,
    including a row pitch that is not a multiple of four and a padded one."""
    import torch
    for shape, pitch in (((97, 517), 517), ((64, 130), 160)):
        inits = [jacobi_init(shape, seed) for seed in range(10, 15)]
        grids = []
        for u0 in inits:
            if pinned:
                buf = torch.empty((shape[0], pitch), dtype=torch.float32, pin_memory=True).numpy()
            else:
                buf = np.empty((shape[0], pitch), np.float32)
            g = buf[:, :shape[1]]
            g[...] = u0
            grids.append(g)
        res = host_api.jacobi2d_host_batch(grids, 9, 3)
        for k, (g, u0, r) in enumerate(zip(grids, inits, res)):
            want, wres = oracle_mod.jacobi2d(u0, 9, 3)
            assert_bits_equal(g, want, f"batch grid {k} {shape} pitch {pitch}")
            assert np.max(np.abs(r - wres) / np.abs(wres)) <= 1e-12
    # Residual-free batch of one grid equals the single-grid host entry.
    u0 = jacobi_init((33, 40), 21)
    a, b = u0.copy(), u0.copy()
    assert host_api.jacobi2d_host_batch([a], 6) == [None]
    host_api.jacobi2d_host(b, 6, 0)
    assert_bits_equal(a, b, "batch of one vs jacobi2d_host")
    # Zero sweeps: the grids come back unchanged.
    c = u0.copy()
    assert host_api.jacobi2d_host_batch([c, c.copy()], 0) == [None, None]
    assert_bits_equal(c, u0, "zero-sweep batch")
