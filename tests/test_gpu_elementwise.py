"""Elementwise forall maps on the B200 (ewise add, axpy) vs the oracle: bit-exact."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, assert_bits_equal

pytestmark = pytest.mark.gpu

SIZES = [1, 3, 4, 5, 31, 32, 33, 100, 1000, 1024, 10000, 65537, (1 << 20) + 3]


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("n", SIZES)
def test_ewise_matches_oracle(kernels, oracle_mod, n):
    rng = np.random.RandomState(42)
    a = rng.random_sample(n).astype(np.float32)
    b = rng.random_sample(n).astype(np.float32)
    got = kernels.ewise(_t(a), _t(b)).cpu().numpy()
    assert_bits_equal(got, oracle_mod.ewise(a, b), f"ewise n={n}")


def test_ewise_golden_reference_stream(kernels):
    """run_ewise.py test_correctness inputs (RandomState(42)) and its numpy reference."""
    z = np.load(GOLDEN / "ewise.npz")
    for n in z["sizes"]:
        got = kernels.ewise(_t(z[f"A_{n}"]), _t(z[f"B_{n}"])).cpu().numpy()
        assert_bits_equal(got, z[f"C_{n}"], f"golden ewise {n}")
        assert float(np.max(np.abs(got - z[f"C_{n}"]))) < 1e-5  # the reference's tolerance


def test_ewise_strided_and_offset(kernels, oracle_mod):
    import torch
    rng = np.random.RandomState(7)
    base_a = torch.from_numpy(rng.random_sample(3001).astype(np.float32)).cuda()
    base_b = torch.from_numpy(rng.random_sample(2003).astype(np.float32)).cuda()
    a = base_a[1::3]            # stride 3, misaligned start
    b = base_b[3:3 + a.shape[0]]  # unit stride, 12-byte offset
    out = torch.zeros(a.shape[0] * 2, device="cuda")[::2]
    kernels.ewise(a, b, out)
    want = oracle_mod.ewise(a.cpu().numpy(), b.cpu().numpy())
    assert_bits_equal(out.cpu().numpy(), want, "strided ewise")


@pytest.mark.parametrize("n", SIZES)
def test_axpy_matches_oracle(kernels, oracle_mod, n):
    rng = np.random.RandomState(1)
    x = (rng.random_sample(n) * 2 - 1).astype(np.float32)
    y = (rng.random_sample(n) * 2 - 1).astype(np.float32)
    ty = _t(y)
    kernels.axpy(2.5, _t(x), ty)
    assert_bits_equal(ty.cpu().numpy(), oracle_mod.axpy(2.5, x, y), f"axpy n={n}")


def test_axpy_golden(kernels):
    z = np.load(GOLDEN / "axpy.npz")
    ty = _t(z["y"])
    kernels.axpy(2.5, _t(z["x"]), ty)
    assert_bits_equal(ty.cpu().numpy(), z["out"], "golden axpy")


def test_axpy_full_size_against_torch_fp32():
    """N = 2^28 (the axpy config): bit-exact vs torch's separate mul then add
    (two IEEE-rounded f32 ops, the same unfused arithmetic)."""
    import torch
    k = __import__("importlib").import_module("spmd-dialect_b200.kernels")
    g = torch.Generator(device="cuda").manual_seed(1)
    n = 1 << 28
    x = torch.rand(n, device="cuda", generator=g) * 2 - 1
    y = torch.rand(n, device="cuda", generator=g) * 2 - 1
    want = torch.add(torch.mul(x, 2.5), y)
    k.axpy(2.5, x, y)
    assert torch.equal(y.view(torch.int32), want.view(torch.int32))
    del x, y, want
    torch.cuda.empty_cache()


def test_ewise_zero_length_is_noop(kernels):
    import torch
    a = torch.empty(0, device="cuda")
    out = kernels.ewise(a, a)
    assert out.numel() == 0
