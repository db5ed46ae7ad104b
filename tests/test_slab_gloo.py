"""Host logic of the multi-GPU row-slab Jacobi-2D, on CPU ranks (gloo).

* partition / neighbours / local_row_range cover every global row exactly once;
* the slab protocol (sweep the owned rows of a (rows+2)-row local array, hand
  the first/last owned row to the neighbours' halo rows, all-gather the
  residual and sum it in rank order) reproduces the single-domain oracle
  bit for bit -- the oracle does each rank's sweep, gloo carries the halos;
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
                assert (lo, hi) == (g0 - 1, g0 + rows + 1)
                up, dn = slab.neighbours(G, world, r)
                assert up == (r - 1 if r else None) and dn == (r + 1 if r < world - 1 else None)
            assert seen == list(range(G))
    with pytest.raises(ValueError):
        slab.partition(3, 4, 0)


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
    u0 = jacobi_init((G, W), 4)
    g0, rows = slab.partition(G, world, rank)
    lo, hi = slab.local_row_range(G, world, rank)
    u = np.zeros((rows + 2, W), np.float32)
    u[max(lo, 0) - lo:min(hi, G) - lo] = u0[max(lo, 0):min(hi, G)]
    v = np.zeros_like(u)
    up, dn = slab.neighbours(G, world, rank)
    res = []
    for k in range(1, sweeps + 1):
        want = res_every > 0 and k % res_every == 0
        rr = oracle.jacobi2d_rows(u, v, 1, rows + 1, g0 - 1, G, want_res=want)
        # halo hand-off: first owned row up, last owned row down
        reqs = []
        if up is not None:
            reqs.append(dist.isend(torch.from_numpy(v[1].copy()), up, tag=2 * k))
            buf = torch.empty(W)
            dist.recv(buf, up, tag=2 * k + 1)
            v[0] = buf.numpy()
        if dn is not None:
            reqs.append(dist.isend(torch.from_numpy(v[rows].copy()), dn, tag=2 * k + 1))
            buf = torch.empty(W)
            dist.recv(buf, dn, tag=2 * k)
            v[rows + 1] = buf.numpy()
        for r in reqs:
            r.wait()
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
        u, v = v, u
    parts = [None] * world
    dist.all_gather_object(parts, u[1:rows + 1])
    if rank == 0:
        q.put((np.concatenate(parts, 0), np.array(res)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,G,W,sweeps", [(2, 37, 29, 7), (3, 64, 17, 5), (2, 3, 8, 3)])
def test_slab_protocol_matches_single_domain_oracle(oracle_mod, world, G, W, sweeps):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_slab_worker, args=(r, world, port, G, W, sweeps, 1, q)) for r in range(world)]
    for p in ps:
        p.start()
    grid, res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    want, wres = oracle_mod.jacobi2d(jacobi_init((G, W), 4), sweeps, 1)
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
