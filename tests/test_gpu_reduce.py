"""spmd.reduce add on the B200 vs the oracle.

f32: within 1e-6 relative of the f64 sum (the target tolerance; the
reference's own check is 1e-3 against np.sum, run_reduction.py:137-141), and
bitwise identical across calls.  i32: exact.  Mirrors the reference's
hierarchical suite: sizes 1..2^24, zeros, ones, 3x multi-launch and the
negative double-accumulation self-test (run_reduction.py:161-264)."""
from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN, spmd_mod

pytestmark = pytest.mark.gpu

REL_F32 = 1e-6
RED = json.loads((GOLDEN / "reduction.json").read_text())


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _zero_out():
    import torch
    return torch.zeros(1, dtype=torch.float32, device="cuda")


def test_hierarchical_suite_sizes(kernels, oracle_mod):
    rng = np.random.RandomState(0)
    for n, np_sum, f64 in zip(RED["sizes"], RED["np_sum"], RED["f64_sum"]):
        a = rng.random_sample(n).astype(np.float32)
        ta = _t(a)
        got = float(kernels.sum_f32(ta, _zero_out()).item())
        assert abs(got - f64) / f64 <= REL_F32, f"n={n}: {got} vs {f64}"
        assert abs(got - np_sum) / max(abs(np_sum), 1e-6) < 1e-3
        # the reference-semantics entry (one f32 atomic per block)
        got_h = float(kernels.hierarchical_sum(ta, _zero_out()).item())
        assert abs(got_h - np_sum) / max(abs(np_sum), 1e-6) < 1e-3
        assert abs(got_h - f64) / f64 <= 1e-5


def test_f32_sum_config_full_size(kernels):
    """N = 2^24 from seed 0 (the reduction config)."""
    a = np.random.RandomState(0).random_sample(1 << 24).astype(np.float32)
    assert hashlib.sha256(a.tobytes()).hexdigest() == RED["f32_cfg_sha256"]
    ta = _t(a)
    ws = kernels.sum_workspace(a.size)
    vals = [float(kernels.sum_f32(ta, _zero_out(), ws).item()) for _ in range(3)]
    f64 = RED["f32_cfg_f64_sum"]
    assert abs(vals[0] - f64) / f64 <= REL_F32
    assert vals[0] == vals[1] == vals[2], "sum_f32 must be deterministic"
    # single rounding: the result is the f32 nearest to the f64 sum (ties aside)
    assert abs(vals[0] - f64) <= abs(float(np.nextafter(np.float32(vals[0]), np.float32(np.inf))) - vals[0])


def test_known_answers(kernels):
    for n in (256, 1024):
        assert float(kernels.sum_f32(_t(np.zeros(n, np.float32)), _zero_out()).item()) == 0.0
        assert float(kernels.sum_f32(_t(np.ones(n, np.float32)), _zero_out()).item()) == float(n)
    assert float(kernels.sum_f32(_t(np.zeros(0, np.float32)), _zero_out()).item()) == 0.0


def test_multi_launch(kernels):
    rng = np.random.RandomState(0)
    for n in RED["sizes"]:
        rng.random_sample(n)  # advance the stream exactly as the reference suite does
    a = rng.random_sample(65536).astype(np.float32)
    assert hashlib.sha256(a.tobytes()).hexdigest() == RED["multi_sha256"]
    ta = _t(a)
    ws = kernels.sum_workspace(a.size)
    for _ in range(3):
        got = float(kernels.sum_f32(ta, _zero_out(), ws).item())
        assert abs(got - RED["multi_f64_sum"]) / RED["multi_f64_sum"] <= REL_F32


def test_negative_double_accumulation_detected(kernels):
    """Two launches without re-zeroing accumulate ~2x: the check must FAIL."""
    a = np.random.RandomState(99).random_sample(1024).astype(np.float32)
    ta = _t(a)
    out = _zero_out()
    kernels.sum_f32(ta, out)
    kernels.sum_f32(ta, out)
    got = float(out.item())
    ref = RED["negative_f64_sum"]
    assert abs(got - ref) / ref >= 1e-3
    assert abs(got - 2 * ref) / (2 * ref) <= REL_F32


def test_strided_sum(kernels, oracle_mod):
    import torch
    base = torch.from_numpy(np.random.RandomState(5).random_sample(30001).astype(np.float32)).cuda()
    a = base[1::3]
    got = float(kernels.sum_f32(a, _zero_out()).item())
    want = oracle_mod.sum_f64(a.cpu().numpy())
    assert abs(got - want) / want <= REL_F32


@pytest.mark.parametrize("n", [1, 7, 1000, 65537, 1 << 24])
def test_i32_sum_exact(kernels, oracle_mod, n):
    import torch
    a = np.random.RandomState(0).randint(0, 100, n, dtype=np.int32)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    kernels.sum_i32(_t(a), out)
    assert int(out.item()) == oracle_mod.sum_i32(a)
    if n == 1 << 24:
        assert hashlib.sha256(a.tobytes()).hexdigest() == RED["i32_sha256"]
        assert int(out.item()) == RED["i32_sum"]


def test_i32_sum_wraps_like_addi(kernels, oracle_mod):
    import torch
    a = np.array([2**31 - 1] * 1000 + [-5, 17], dtype=np.int32)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    kernels.sum_i32(_t(a), out)
    assert int(out.item()) == oracle_mod.sum_i32(a)


def test_partial_sum_is_the_unrounded_f64_total(kernels, oracle_mod):
    """spmdb200_sum_f32_partial: f64 total of a rank's block, both kernel paths."""
    import torch
    shard = spmd_mod("shard")
    for n, stride in ((1 << 20, 1), (100003, 1), (77777, 3)):
        x = np.random.RandomState(n).random_sample(n * stride).astype(np.float32)
        t = torch.from_numpy(x).cuda()[::stride]
        p = float(shard.partial_sum_f32(t).item())
        exact = oracle_mod.sum_f64(np.ascontiguousarray(x[::stride]))
        assert abs(p - exact) <= 1e-12 * abs(exact)
        assert shard.sum_f32(t, init=1.0) == np.float32(1.0 + p)


def test_shared_workspace_stays_zero_across_entries(kernels, oracle_mod):
    """One workspace serves the staged sum, the strided sum and every reduce
    kind.  The staged sum reads a non-zero partial word as written, so every
    entry must leave the workspace all-zero; interleaving them on one
    workspace must not change any result."""
    import torch
    from conftest import spmd_pkg

    a = np.random.RandomState(7).random_sample((1 << 20) + 3).astype(np.float32)
    ia = np.random.RandomState(8).randint(-1000, 1000, 70001, dtype=np.int32)
    ta, tia = _t(a), _t(ia)
    ws = kernels.sum_workspace(a.size)
    f64 = oracle_mod.sum_f64(a)

    def staged():
        v = float(kernels.sum_f32(ta, _zero_out(), ws).item())
        assert abs(v - f64) / f64 <= REL_F32
        return v

    first = staged()
    assert int(torch.count_nonzero(ws)) == 0
    strided = float(kernels.sum_f32(ta[::2], _zero_out(), ws).item())
    want = oracle_mod.sum_f64(a[::2])
    assert abs(strided - want) / want <= REL_F32
    assert int(torch.count_nonzero(ws)) == 0
    assert float(kernels.reduce("max", ta, -1.0, ws=ws).item()) == float(a.max())
    assert int(torch.count_nonzero(ws)) == 0
    got_add = float(kernels.reduce("add", ta, 0.0, ws=ws).item())
    assert abs(got_add - f64) / f64 <= REL_F32
    assert int(torch.count_nonzero(ws)) == 0
    x = int(np.bitwise_xor.reduce(ia))
    assert int(kernels.reduce("xor", tia, 0, ws=ws).item()) == x
    assert int(torch.count_nonzero(ws)) == 0
    assert staged() == first
    assert int(torch.count_nonzero(ws)) == 0
    assert spmd_pkg().lib().spmdb200_reduction_status() == 0
