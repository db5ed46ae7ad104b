"""Host logic of the multi-GPU row-slab Jacobi-2D, on CPU ranks (gloo).

* partition / neighbours / local_row_range cover every global row exactly once;
* the slab protocol (passes of one, two, four or eight sweeps over a
  (rows+16)-row local array -- sweep f of an F-sweep pass also re-sweeps
  F-1-f halo rows on each side --, the first/last eight owned rows handed to
  the neighbours' halo rows after each pass, the residual all-gathered and
  summed in rank order) reproduces the single-domain oracle bit for bit -- the
  oracle does each rank's sweeps, gloo carries the halos;
* a rank that never reaches the rendezvous makes the other rank fail there
  (process-group timeout) instead of proceeding to a launch.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT, jacobi_init, spmd_mod


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_covers_rows_once():
    slab = spmd_mod("slab")
    for G in (2, 3, 7, 64, 1001):
        for world in (1, 2, 3, 4, 8):
            if G < world:
                continue
            seen = []
            for r in range(world):
                g0, rows = slab.partition(G, world, r)
                assert rows >= 1
                seen.extend(range(g0, g0 + rows))
                lo, hi = slab.local_row_range(G, world, r)
                assert (lo, hi) == (g0 - slab.HALO, g0 + rows + slab.HALO)
                up, dn = slab.neighbours(G, world, r)
                assert up == (r - 1 if r else None) and dn == (r + 1 if r < world - 1 else None)
            assert seen == list(range(G))
    with pytest.raises(ValueError):
        slab.partition(3, 4, 0)


def _pass_plan(sweeps: int, res_every: int, fmax: int = 8) -> list[int]:
    """Sweeps per pass as the C library schedules them: even numbers of
    eight- (2-D only), four- and two-sweep passes (none longer than the
    residual interval), then the single sweeps left over."""
    top = fmax
    while res_every > 0 and fmax > res_every:
        fmax //= 2
    plan, left = [], sweeps
    for f in [x for x in (8, 4, 2, 1) if x <= top]:
        n = 0 if f > fmax else left if f == 1 else (left // (2 * f)) * 2
        plan += [f] * n
        left -= n * f
    return plan


def _slab_worker(rank: int, world: int, port: int, G: int, W: int, sweeps: int, res_every: int, q):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch
    import torch.distributed as dist
    from oracle import oracle
    from conftest import spmd_mod as _m
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    slab = _m("slab")
    H = slab.HALO
    u0 = jacobi_init((G, W), 4)
    g0, rows = slab.partition(G, world, rank)
    lo, hi = slab.local_row_range(G, world, rank)
    u = np.zeros((rows + 2 * H, W), np.float32)
    u[max(lo, 0) - lo:min(hi, G) - lo] = u0[max(lo, 0):min(hi, G)]
    v = np.zeros_like(u)
    up, dn = slab.neighbours(G, world, rank)
    res = []
    k = 0
    for pno, F in enumerate(_pass_plan(sweeps, res_every)):
        # Sweep f of an F-sweep pass also sweeps F-1-f halo rows beyond each
        # edge (the later sweeps of the owned edge rows read them).
        for f in range(F):
            k += 1
            want = res_every > 0 and k % res_every == 0
            ext = F - 1 - f
            src, dst = (u, v) if f % 2 == 0 else (v, u)
            oracle.jacobi2d_rows(src, dst, H - ext, H + rows + ext, g0 - H, G)
            rr = oracle.jacobi2d_rows(src, dst, H, H + rows, g0 - H, G, want_res=True) if want else None
            if want:
                mine = 0.0
                for x in rr:
                    mine = mine + float(x)
                slots = [None] * world
                dist.all_gather_object(slots, mine)
                tot = 0.0
                for x in slots:  # rank order, as spmdb200_jacobi2d_slab_residuals sums
                    tot = tot + x
                res.append(tot)
        out = v if F % 2 == 1 else u
        # halo hand-off after each pass: the first H owned rows up, the last H down
        reqs = []
        if up is not None:
            reqs.append(dist.isend(torch.from_numpy(out[H:2 * H].copy()), up, tag=2 * pno))
            buf = torch.empty((H, W))
            dist.recv(buf, up, tag=2 * pno + 1)
            out[0:H] = buf.numpy()
        if dn is not None:
            reqs.append(dist.isend(torch.from_numpy(out[rows:rows + H].copy()), dn, tag=2 * pno + 1))
            buf = torch.empty((H, W))
            dist.recv(buf, dn, tag=2 * pno)
            out[rows + H:rows + 2 * H] = buf.numpy()
        for r in reqs:
            r.wait()
        if F % 2 == 1:
            u, v = v, u
    parts = [None] * world
    dist.all_gather_object(parts, u[H:rows + H])
    if rank == 0:
        q.put((np.concatenate(parts, 0), np.array(res)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,G,W,sweeps,res_every", [(2, 37, 29, 7, 1), (3, 64, 17, 5, 2), (2, 16, 8, 3, 1),
                                                         (2, 37, 29, 20, 10), (4, 41, 13, 19, 8),
                                                         (2, 50, 21, 22, 0), (3, 40, 9, 17, 4)])
def test_slab_protocol_matches_single_domain_oracle(oracle_mod, world, G, W, sweeps, res_every):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_slab_worker, args=(r, world, port, G, W, sweeps, res_every, q)) for r in range(world)]
    for p in ps:
        p.start()
    grid, res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    want, wres = oracle_mod.jacobi2d(jacobi_init((G, W), 4), sweeps, res_every)
    assert np.array_equal(grid.view(np.uint32), want.view(np.uint32))
    np.testing.assert_allclose(res, wres, rtol=1e-12)


def _zslab_worker(rank: int, world: int, port: int, D: int, H: int, W: int, sweeps: int, res_every: int, q):
    """Jacobi-3D z-slab protocol: passes of up to HALO3 sweeps over a
    (planes + 2 HALO3)-plane local array -- sweep f of an F-sweep pass also re-sweeps
    F-1-f halo planes on each side --, the first/last F owned planes handed to
    the neighbours' halo planes after each pass, residuals summed in rank
    order."""
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch
    import torch.distributed as dist
    from oracle import oracle
    from conftest import spmd_mod as _m
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    slab = _m("slab")
    h = slab.HALO3
    u0 = jacobi_init((D, H, W), 3)
    z0, planes = slab.partition(D, world, rank)
    lo, hi = z0 - h, z0 + planes + h
    u = np.zeros((planes + 2 * h, H, W), np.float32)
    u[max(lo, 0) - lo:min(hi, D) - lo] = u0[max(lo, 0):min(hi, D)]
    v = np.zeros_like(u)
    up, dn = slab.neighbours(D, world, rank)
    res = []
    k = 0
    for pno, F in enumerate(_pass_plan(sweeps, res_every, fmax=h)):
        for f in range(F):
            k += 1
            want = res_every > 0 and k % res_every == 0
            ext = F - 1 - f
            src, dst = (u, v) if f % 2 == 0 else (v, u)
            oracle.jacobi3d_planes(src, dst, h - ext, h + planes + ext, z0 - h, D)
            pr = oracle.jacobi3d_planes(src, dst, h, h + planes, z0 - h, D, want_res=True) if want else None
            if want:
                mine = 0.0
                for x in pr:
                    mine = mine + float(x)
                slots = [None] * world
                dist.all_gather_object(slots, mine)
                tot = 0.0
                for x in slots:
                    tot = tot + x
                res.append(tot)
        out = v if F % 2 == 1 else u
        # halo hand-off after each pass: the first F owned planes up, the last F down
        reqs = []
        if up is not None:
            reqs.append(dist.isend(torch.from_numpy(out[h:h + F].copy()), up, tag=2 * pno))
            buf = torch.empty((F, H, W))
            dist.recv(buf, up, tag=2 * pno + 1)
            out[h - F:h] = buf.numpy()
        if dn is not None:
            reqs.append(dist.isend(torch.from_numpy(out[h + planes - F:h + planes].copy()), dn, tag=2 * pno + 1))
            buf = torch.empty((F, H, W))
            dist.recv(buf, dn, tag=2 * pno)
            out[h + planes:h + planes + F] = buf.numpy()
        for r in reqs:
            r.wait()
        if F % 2 == 1:
            u, v = v, u
    parts = [None] * world
    dist.all_gather_object(parts, u[h:h + planes])
    if rank == 0:
        q.put((np.concatenate(parts, 0), np.array(res)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,D,H,W,sweeps,res_every", [(2, 9, 6, 7, 5, 1), (3, 13, 5, 9, 4, 2),
                                                           (4, 17, 3, 5, 9, 0), (2, 11, 6, 10, 13, 4),
                                                           (3, 20, 5, 6, 11, 3)])
def test_zslab_protocol_matches_single_domain_oracle(oracle_mod, world, D, H, W, sweeps, res_every):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_zslab_worker, args=(r, world, port, D, H, W, sweeps, res_every, q))
          for r in range(world)]
    for p in ps:
        p.start()
    grid, res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    want, wres = oracle_mod.jacobi3d(jacobi_init((D, H, W), 3), sweeps, res_every)
    assert np.array_equal(grid.view(np.uint32), want.view(np.uint32))
    np.testing.assert_allclose(res, wres, rtol=1e-12)


def _dead_rank_worker(rank: int, port: int, q):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    from datetime import timedelta

    import torch.distributed as dist
    from conftest import spmd_mod as _m
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # dies between steps, before the next launch's rendezvous
    try:
        _m("slab").rendezvous()
        q.put("passed")
    except Exception as e:  # noqa: BLE001 -- the failure is the expected outcome
        q.put(f"raised {type(e).__name__}")


def test_dead_rank_detected_at_rendezvous():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dead_rank_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
    assert out.startswith("raised"), out
