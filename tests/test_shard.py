"""Host logic of the 1-D operations split across GPUs: block ranges, the
rank-order f32 combine and the wrapping int32 combine (CPU only)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import spmd_mod


def test_shard_range_covers_once():
    sh = spmd_mod("shard")
    for n in (0, 1, 7, 1000, 2 ** 24 + 3):
        for world in (1, 2, 3, 8):
            got = [sh.shard_range(n, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            assert max(h - l for l, h in got) - min(h - l for l, h in got) <= 1
    with pytest.raises(ValueError):
        sh.shard_range(10, 2, 2)


def test_combine_f32_rounds_once_in_rank_order():
    sh = spmd_mod("shard")
    parts = [1e8, 1.0, -1e8, 0.25]
    want = np.float32(float(np.float32(0.5)) + (((1e8 + 1.0) + -1e8) + 0.25))
    assert sh.combine_f32(parts, 0.5) == want
    x = np.random.RandomState(0).random_sample(10001).astype(np.float32)
    blocks = [x[lo:hi].astype(np.float64).sum() for lo, hi in (sh.shard_range(x.size, 3, r) for r in range(3))]
    exact = x.astype(np.float64).sum()
    assert abs(float(sh.combine_f32(blocks)) - exact) <= 1e-6 * exact


def test_combine_i32_wraps_like_the_single_gpu_sum():
    sh = spmd_mod("shard")
    v = np.random.RandomState(1).randint(-2 ** 31, 2 ** 31, size=5000, dtype=np.int64).astype(np.int32)
    totals = []
    for r in range(4):
        lo, hi = sh.shard_range(v.size, 4, r)
        totals.append(int(v[lo:hi].astype(np.int64).sum()))
    want = int(v.sum(dtype=np.int32))  # numpy wraps in int32
    assert sh.combine_i32(totals) == want
    assert sh.combine_i32([2 ** 31 - 1], 1) == -2 ** 31
