"""Checkpoint file format (host only): header round trip, block-wise writes by
several writers (the slab ranks), reads with halos past the grid edges, and
resume semantics on the oracle (k sweeps, save, load, m sweeps == k + m)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import jacobi_init, spmd_mod


def test_header_round_trip(tmp_path):
    ck = spmd_mod("checkpoint")
    p = str(tmp_path / "a.ckpt")
    ck.write_header(p, (5, 7, 3), sweeps=123, res_every=10)
    info = ck.read_header(p)
    assert info.shape == (5, 7, 3) and info.sweeps == 123 and info.res_every == 10
    assert (tmp_path / "a.ckpt").stat().st_size == ck.HEADER + 4 * 5 * 7 * 3


def test_rejects_foreign_and_truncated_files(tmp_path):
    ck = spmd_mod("checkpoint")
    bad = tmp_path / "bad.ckpt"
    bad.write_bytes(b"NOTACKPT" + bytes(56) + bytes(16))
    with pytest.raises(ValueError):
        ck.read_header(str(bad))
    p = str(tmp_path / "t.ckpt")
    ck.write_header(p, (4, 4), sweeps=0)
    with open(p, "r+b") as f:
        f.truncate(ck.HEADER + 10)
    with pytest.raises(ValueError):
        ck.read_header(p)
    with pytest.raises(ValueError):
        ck.write_header(p, (4,), sweeps=0)


def test_blocks_from_several_writers_and_halo_reads(tmp_path):
    ck = spmd_mod("checkpoint")
    slab = spmd_mod("slab")
    g = np.random.RandomState(0).random_sample((37, 11)).astype(np.float32)
    p = str(tmp_path / "g.ckpt")
    ck.write_header(p, g.shape, sweeps=9)
    for r in range(3):  # three "ranks" write their own rows
        g0, rows = slab.partition(37, 3, r)
        ck.write_block(p, g0, g[g0:g0 + rows])
    back, info = ck.load_grid(p)
    assert np.array_equal(back, g) and info.sweeps == 9
    # a rank's rows with 4 halo rows each side; rows outside the grid are 0
    blk = ck.read_block(p, -4, 9)
    assert np.array_equal(blk[4:], g[:9]) and not blk[:4].any()
    blk = ck.read_block(p, 30, 41)
    assert np.array_equal(blk[:7], g[30:]) and not blk[7:].any()
    with pytest.raises(ValueError):
        ck.write_block(p, 35, g[:5])


def test_resume_equals_uninterrupted_run(tmp_path, oracle_mod):
    ck = spmd_mod("checkpoint")
    u0 = jacobi_init((40, 33), 4)
    mid, _ = oracle_mod.jacobi2d(u0, 7, 0)
    p = str(tmp_path / "j.ckpt")
    ck.save_grid(p, mid, sweeps=7)
    back, info = ck.load_grid(p)
    fin, _ = oracle_mod.jacobi2d(back, 6, 0)
    want, _ = oracle_mod.jacobi2d(u0, 13, 0)
    assert info.sweeps == 7
    assert np.array_equal(fin.view(np.uint32), want.view(np.uint32))
    u3 = jacobi_init((9, 8, 10), 3)
    mid3, _ = oracle_mod.jacobi3d(u3, 3, 0)
    p3 = str(tmp_path / "j3.ckpt")
    ck.save_grid(p3, mid3, sweeps=3)
    back3, info3 = ck.load_grid(p3)
    assert info3.shape == (9, 8, 10)
    fin3, _ = oracle_mod.jacobi3d(back3, 2, 0)
    want3, _ = oracle_mod.jacobi3d(u3, 5, 0)
    assert np.array_equal(fin3.view(np.uint32), want3.view(np.uint32))
