"""The general promoted-tile stencil (spmdb200_stencil_nd) on the GPU against
the oracle (oracle_stencil_nd), bit for bit: ranks 1-3, steps, positive- and
negative-only halos, weights and a final scale, ragged sizes, the reference's
promoted 3-point stencil and the Jacobi interiors as special cases, and the
promoted and direct paths giving identical results."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_bits_equal, spmd_mod

pytestmark = pytest.mark.gpu

THREE_POINT = [[0, 0], [0, 1], [1, 0]]  # (A[i,j] + A[i,j+1]) + A[i+1,j]
JACOBI5 = [[0, 0], [-1, 0], [1, 0], [0, 1], [0, -1]]  # ((((c + n) + s) + e) + w)
JACOBI7 = [[0, 0, 0], [0, 0, -1], [0, 0, 1], [0, -1, 0], [0, 1, 0], [-1, 0, 0], [1, 0, 0]]


def _rand(shape, seed):
    return np.random.RandomState(seed).random_sample(shape).astype(np.float32)


def _run(kernels, a, out_shape, offsets, weights=None, scale=1.0, tile=None, steps=None, policy=0, mgb=0, init=None):
    ta = torch.from_numpy(a).cuda()
    tb = torch.zeros(out_shape, device="cuda") if init is None else torch.from_numpy(init).cuda()
    promoted = kernels.stencil_nd(ta, tb, offsets, weights=weights, scale=scale, tile_sizes=tile, steps=steps,
                                  policy=policy, max_group_bytes=mgb)
    torch.cuda.synchronize()
    return tb.cpu().numpy(), promoted


@pytest.mark.parametrize("n,m", [(64, 64), (511, 513), (33, 9), (1, 1), (100, 7)])
def test_three_point_is_the_promoted_stencil(kernels, oracle_mod, n, m):
    a = _rand((n + 1, m + 1), 0)
    got, promoted = _run(kernels, a, (n, m), THREE_POINT, tile=[32, 8])
    assert promoted, "33x9 footprint must be promoted"
    assert_bits_equal(got, oracle_mod.stencil3(a, n, m), "stencil_nd 3-point vs stencil_cpu")


@pytest.mark.parametrize("policy", [0, 1])
def test_jacobi5_interior(kernels, oracle_mod, policy):
    u = _rand((130, 260), 2)
    got, promoted = _run(kernels, u, u.shape, JACOBI5, scale=0.2, tile=[16, 32], policy=policy)
    assert promoted == (policy == 0)
    want = oracle_mod.stencil_nd(u, u.shape, JACOBI5, scale=0.2)
    assert_bits_equal(got, want)
    one, _ = oracle_mod.jacobi2d(u, 1, 0)  # interior cells equal one Jacobi sweep
    assert_bits_equal(got[1:-1, 1:-1], one[1:-1, 1:-1], "interior vs jacobi2d")


def test_jacobi7_interior_3d(kernels, oracle_mod):
    u = _rand((20, 17, 40), 3)
    got, promoted = _run(kernels, u, u.shape, JACOBI7, scale=np.float32(1.0 / 7.0), tile=[4, 8, 32])
    assert promoted
    one, _ = oracle_mod.jacobi3d(u, 1, 0)
    assert_bits_equal(got[1:-1, 1:-1, 1:-1], one[1:-1, 1:-1, 1:-1], "interior vs jacobi3d")


@pytest.mark.parametrize("offs,steps", [([[0], [1]], [2]), ([[1], [2]], None), ([[-2], [-1]], None)])
def test_1d_stepped_and_one_sided_halos(kernels, oracle_mod, offs, steps):
    a = _rand(1003, 5)
    init = _rand(1001, 6)  # points off the step lattice must stay untouched
    got, promoted = _run(kernels, a, (1001,), offs, tile=[4], steps=steps, init=init)
    assert promoted
    assert_bits_equal(got, oracle_mod.stencil_nd(a, (1001,), offs, steps=steps, out=init))


@pytest.mark.parametrize("rank,shape_a,shape_b,tile,seed", [
    (2, (77, 91), (80, 90), [16, 16], 7),
    (3, (9, 13, 70), (10, 12, 66), [2, 4, 32], 8),
    (1, (5000,), (4999,), [128], 9),
])
def test_random_weighted_taps(kernels, oracle_mod, rank, shape_a, shape_b, tile, seed):
    rng = np.random.RandomState(seed)
    offs = rng.randint(-2, 3, size=(9, rank)).tolist()
    w = rng.random_sample(9).astype(np.float32) * 2 - 1
    a = _rand(shape_a, seed)
    got, _ = _run(kernels, a, shape_b, offs, weights=w.tolist(), scale=0.75, tile=tile)
    want = oracle_mod.stencil_nd(a, shape_b, offs, weights=w, scale=0.75)
    assert_bits_equal(got, want)
    direct, promoted = _run(kernels, a, shape_b, offs, weights=w.tolist(), scale=0.75, tile=tile, policy=1)
    assert not promoted
    assert_bits_equal(direct, want, "direct path")


def test_oversized_footprint_falls_back_and_limit_override(kernels, oracle_mod):
    a = _rand((300, 300), 11)
    got, promoted = _run(kernels, a, (299, 299), THREE_POINT, tile=[128, 128])
    assert not promoted  # 129 x 129 x 4 B > 48 KB
    want = oracle_mod.stencil3(a, 299, 299)
    assert_bits_equal(got, want)
    got2, promoted2 = _run(kernels, a, (299, 299), THREE_POINT, tile=[128, 128], mgb=96 * 1024)
    assert promoted2
    assert_bits_equal(got2, want)


def test_rejects_overlap_and_bad_arguments(kernels):
    L = spmd_mod("_lib")
    t = torch.zeros((64, 64), device="cuda")
    with pytest.raises(L.SpmdError):
        kernels.stencil_nd(t, t, THREE_POINT)
    with pytest.raises(L.SpmdError):
        kernels.stencil_nd(t, torch.zeros((64, 64), device="cuda"), [[0, 0]] * 65)


@pytest.mark.parametrize("shape,offsets,weights,steps,shift", [
    ((9, 20, 140), JACOBI7, None, None, 0),                                       # one ring of 4 planes
    ((13, 7, 33), [[2, 1, -3], [-3, 0, 2], [0, 0, 0]], [0.5, 0.25, 2.0], None, 1),  # z span 5: ring of 8
    ((30, 18, 40), [[0, 0, 0], [1, 1, 1]], None, [1, 2, 1], 2),                    # y step 2
    ((5, 3, 6), [[6, 0, 0], [0, 0, 0]], None, None, 3),                           # z span 6, planes past A
    ((70, 37, 261), JACOBI7, None, None, 1),                                      # several z items, ragged x
    ((6, 5, 512), JACOBI7, None, None, 2),                                        # 256-point row segments
    ((11, 9, 1030), [[0, 0, 0], [1, -1, 2], [-1, 1, -2]], [1.0, -0.5, 0.5], None, 3),  # 256-point, ragged
])
def test_rank3_z_streaming(kernels, oracle_mod, shape, offsets, weights, steps, shift):
    """Rank 3, unit strides, z step 1: the z-streaming kernel (a ring of
    planes), A starting at every 4-byte phase of a 16-byte line."""
    base = torch.from_numpy(_rand(int(np.prod(shape)) + 3, 11)).cuda()
    ta = base[shift:shift + int(np.prod(shape))].view(shape)
    b_shape = tuple(shape)
    tb = torch.zeros(b_shape, device="cuda")
    scale = np.float32(1.0 / 7.0) if offsets is JACOBI7 else 1.0
    promoted = kernels.stencil_nd(ta, tb, offsets, weights=weights, scale=scale, tile_sizes=[2, 4, 8], steps=steps)
    torch.cuda.synchronize()
    assert promoted
    want = oracle_mod.stencil_nd(ta.cpu().numpy(), b_shape, offsets, weights=weights, scale=scale, steps=steps)
    assert_bits_equal(tb.cpu().numpy(), want, f"z-streaming {shape}")
