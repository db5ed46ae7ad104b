"""The general elementwise forall (spmdb200_forall_map) on the GPU against the
oracle: random body programs over every opcode, rank 1-3, ragged sizes,
strided / misaligned / in-place views, and the shim's MLIR kernels called with
their own argument lists.  Bit-exact, except that a NaN matches any NaN
(payloads are not specified)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ROOT, spmd_mod
from test_forall_program import bits_equal_nan, random_dag

pytestmark = pytest.mark.gpu
fp = spmd_mod("forall_program")


def _check(got: np.ndarray, want: np.ndarray, what: str):
    assert got.shape == want.shape, what
    if not bits_equal_nan(got, want):
        ng, nw = np.isnan(got), np.isnan(want)
        bad = np.nonzero((got.view(np.uint32) != want.view(np.uint32)) & ~(ng & nw))
        idx = tuple(x[0] for x in bad)
        raise AssertionError(f"{what}: {bad[0].size} points differ; first at {idx}: {got[idx]!r} vs {want[idx]!r}")


SHAPES = [(1,), (7,), (2049,), (1 << 16,), (3, 5), (37, 129), (256, 1000), (2, 3, 4), (5, 17, 33), (16, 64, 96)]


@pytest.mark.parametrize("seed", range(16))
def test_random_programs_match_oracle(kernels, oracle_mod, seed):
    rs = np.random.RandomState(500 + seed)
    n_in = 1 + seed % 5
    root, nodes, consts = random_dag(rs, n_in, 3 + 2 * (seed % 7))
    code, n_regs, _, _ = fp.compile_dag(root, nodes)
    shape = SHAPES[seed % len(SHAPES)]
    ins = [rs.uniform(-4, 4, size=shape).astype(np.float32) for _ in range(n_in)]
    flat = ins[0].reshape(-1)
    flat[: min(4, flat.size)] = [0.0, -0.0, np.inf, -np.inf][: min(4, flat.size)]
    want = oracle_mod.forall_map(ins, shape, code, consts)
    out = torch.full(shape, 7.0, device="cuda")
    kernels.forall_map([torch.from_numpy(a).cuda() for a in ins], out, code, consts, n_regs=n_regs)
    _check(out.cpu().numpy(), want, f"seed {seed} shape {shape}")


def test_every_cmpf_predicate_with_nans(kernels, oracle_mod):
    rs = np.random.RandomState(9)
    a = rs.choice(np.array([0.0, -0.0, 1.0, -1.0, np.nan, np.inf, -np.inf], np.float32), size=4099)
    b = rs.choice(np.array([0.0, 1.0, np.nan, -np.inf], np.float32), size=4099)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    for pred in range(16):
        nodes = {"a": ("load", 0), "b": ("load", 1), "c": ("cmp", "a", "b", pred), "m": ("maximum", "a", "b"),
                 "n": ("minimum", "a", "b"), "s": ("select", "c", "m", "n")}
        code, n_regs, _, _ = fp.compile_dag("s", nodes)
        out = torch.empty(4099, device="cuda")
        kernels.forall_map([ta, tb], out, code, n_regs=n_regs)
        _check(out.cpu().numpy(), oracle_mod.forall_map([a, b], a.shape, code), f"predicate {pred}")


def test_strided_misaligned_and_in_place_views(kernels, oracle_mod):
    rs = np.random.RandomState(11)
    nodes = {"a": ("load", 0), "b": ("load", 1), "c": ("const", 0), "p": ("mul", "a", "b"), "q": ("add", "p", "c"),
             "r": ("div", "q", "b")}
    code, n_regs, _, _ = fp.compile_dag("r", nodes)
    base = rs.uniform(0.5, 2, size=(70, 90)).astype(np.float32)
    other = rs.uniform(0.5, 2, size=(90, 70)).astype(np.float32)
    tb, to = torch.from_numpy(base).cuda(), torch.from_numpy(other).cuda()
    flat, flat2 = tb.reshape(-1), to.reshape(-1)
    views = [
        ("transposed", tb[:64, :64], to.t()[:64, :64]),
        ("offset by one", tb[:, 1:65], tb[:, 2:66]),  # 4-byte aligned only
        ("row step 2", tb[::2, :], to.t()[:35, :90]),
        ("short strided rows", tb[:50, :3], to.t()[:50, :3]),  # every group crosses a row end
        ("contiguous, misaligned 1-D", flat[1:4001], flat2[3:4003]),
        ("contiguous, misaligned 2-D", flat[1:1 + 63 * 97].view(63, 97), flat2[2:2 + 63 * 97].view(63, 97)),
        ("contiguous 3-D, one misaligned", flat[:5 * 7 * 11].view(5, 7, 11), flat2[1:1 + 385].view(5, 7, 11)),
    ]
    long_a = torch.from_numpy(rs.uniform(0.5, 2, size=(8, 3000)).astype(np.float32)).cuda()
    long_b = torch.from_numpy(rs.uniform(0.5, 2, size=(3, 4, 1600)).astype(np.float32)).cuda()
    views += [
        ("long pitched rows", long_a[:, :2500], long_a[:, 7:2507]),  # rows of >= 1024 points: row chunks
        ("long pitched rows 3-D", long_b[:, :, :1500], long_b[:, :, 100:1600]),
        ("long rows, column step 2", long_a[:, :2400:2], long_a[:, 1:2401:2]),
    ]
    for what, va, vb in views:
        out = torch.zeros(va.shape, device="cuda")
        kernels.forall_map([va, vb], out, code, [0.25], n_regs=n_regs)
        want = oracle_mod.forall_map([va.cpu().numpy(), vb.cpu().numpy()], tuple(va.shape), code, [0.25])
        _check(out.cpu().numpy(), want, what)
    # in place: the output is the first input (same view)
    x = rs.uniform(-1, 1, size=(1 << 20) + 3).astype(np.float32)
    y = rs.uniform(0.5, 1, size=x.size).astype(np.float32)
    tx, ty = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    kernels.forall_map([tx, ty], tx, code, [0.25], n_regs=n_regs)
    _check(tx.cpu().numpy(), oracle_mod.forall_map([x, y], x.shape, code, [0.25]), "in place")


def test_empty_domain_launches_nothing(kernels):
    out = torch.zeros((0, 5), device="cuda")
    kernels.forall_map([torch.zeros((0, 5), device="cuda")], out, [fp.insn("load", 0, aux=0), fp.insn("store", 0, 0)])


def test_large_contiguous_body(kernels, oracle_mod):
    """2^24 points, three inputs: the 128-bit path across many chunks per block."""
    rs = np.random.RandomState(12)
    n = 1 << 24
    a, b, c = (rs.standard_normal(n).astype(np.float32) for _ in range(3))
    nodes = {"a": ("load", 0), "b": ("load", 1), "c": ("load", 2), "ab": ("mul", "a", "b"), "s": ("sub", "ab", "c"),
             "q": ("abs", "s"), "r": ("sqrt", "q")}
    code, n_regs, _, _ = fp.compile_dag("r", nodes)
    out = torch.empty(n, device="cuda")
    kernels.forall_map([torch.from_numpy(v).cuda() for v in (a, b, c)], out, code, n_regs=n_regs)
    _check(out.cpu().numpy(), oracle_mod.forall_map([a, b, c], (n,), code), "2^24")


@pytest.fixture(scope="module")
def fns(kernels):
    shim = spmd_mod("mlir_shim")
    return shim.load((ROOT / "tests" / "mlir" / "kernels.mlir").read_text(), skip_unmapped=True)


def test_shim_general_bodies(fns):
    rs = np.random.RandomState(13)
    A, B = rs.randn(50, 70).astype(np.float32), rs.randn(50, 70).astype(np.float32)
    C = torch.full((50, 70), -1.0, device="cuda")
    fns["mul2d"](torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), C, 40, 61)
    got = C.cpu().numpy()
    assert np.array_equal(got[:40, :61], A[:40, :61] * B[:40, :61])
    assert (got[40:, :] == -1).all() and (got[:, 61:] == -1).all()
    a = rs.randn(1000).astype(np.float32)
    tb = torch.zeros(1000, device="cuda")
    fns["plus_one_from4"](torch.from_numpy(a).cuda(), tb, 997)
    want = np.zeros(1000, np.float32)
    want[4:997] = a[4:997] + np.float32(1.0)
    assert np.array_equal(tb.cpu().numpy(), want)
    tb = torch.zeros(1000, device="cuda")
    fns["clamp_tiled"](torch.from_numpy(a).cuda(), tb, 1000, 0.75)
    assert np.array_equal(tb.cpu().numpy(), np.clip(a, np.float32(-0.75), np.float32(0.75)))
    X, Y = rs.randn(3, 4, 11).astype(np.float32), rs.randn(3, 4, 11).astype(np.float32)
    R = torch.zeros((3, 4, 11), device="cuda")
    fns["hypot3d"](torch.from_numpy(X).cuda(), torch.from_numpy(Y).cuda(), R, 3, 4, 11)
    xs, ys = X[:, :, ::2], Y[:, :, ::2]
    r = np.sqrt(xs * xs + ys * ys)
    got = R.cpu().numpy()
    assert np.array_equal(got[:, :, ::2], (np.maximum(r, np.abs(xs)) / r).astype(np.float32))
    assert not got[:, :, 1::2].any()
    v = rs.randn(777).astype(np.float32)
    tv = torch.from_numpy(v).cuda()
    fns["scale_in_place"](tv, 777)
    assert np.array_equal(tv.cpu().numpy(), v * np.float32(2.0) + np.float32(1.0))
