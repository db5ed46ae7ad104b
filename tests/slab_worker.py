"""One rank of the 2-GPU slab parity test (launched by test_gpu_slab.py via torchrun).

Every rank builds the same seeded global grid, runs its row slab (Jacobi-2D)
or plane slab (Jacobi-3D) on its own GPU (halo rows / planes stored into the
neighbour over NVLink inside the kernel), and rank 0 compares the gathered
grid and the all-gathered residuals with the single-domain oracle."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def main() -> None:
    import torch
    import torch.distributed as dist

    from conftest import jacobi_init, spmd_mod

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=120))
    slab = spmd_mod("slab")
    rank = dist.get_rank()
    ok = True
    for (G, W, sweeps, res_every) in [(514, 1000, 13, 3), (67, 130, 8, 1), (4096, 4096, 20, 10),
                                      (17, 300, 9, 1), (16, 260, 21, 0)]:  # 9+8 / 8+8 rows: a rank owns one halo's depth
        if G < dist.get_world_size() * slab.HALO:
            continue  # every rank owns at least one halo's depth
        u0 = jacobi_init((G, W), 4)
        job = slab.SlabJacobi2D(cols=W, G=G, res_every=res_every, init=u0)
        job.run(sweeps)
        res = job.residuals()
        grid = job.gather()
        job.close()
        if rank == 0:
            from oracle import oracle
            want, wres = oracle.jacobi2d(u0, sweeps, res_every)
            same = np.array_equal(grid.view(np.uint32), want.view(np.uint32))
            rel = np.max(np.abs(res - wres) / np.abs(wres)) if wres.size else 0.0
            print(f"G={G} W={W} sweeps={sweeps}: grid bit-exact={same} residual max rel err={rel:.3g}", flush=True)
            ok = ok and same and rel <= 1e-12
    # Jacobi-3D z-slabs: HALO3 halo planes each side, passes of up to HALO3 sweeps.
    for (D, H, W, sweeps, res_every) in [(37, 20, 150, 7, 2), (64, 64, 130, 10, 5), (9, 9, 11, 3, 1),
                                         (40, 33, 140, 13, 0), (21, 50, 270, 11, 4)]:
        if D < dist.get_world_size() * slab.HALO3:
            continue
        u0 = jacobi_init((D, H, W), 3)
        job = slab.SlabJacobi3D(H=H, W=W, D=D, res_every=res_every, init=u0)
        job.run(sweeps)
        res = job.residuals()
        grid = job.gather()
        job.close()
        if rank == 0:
            from oracle import oracle
            want, wres = oracle.jacobi3d(u0, sweeps, res_every)
            same = np.array_equal(grid.view(np.uint32), want.view(np.uint32))
            rel = np.max(np.abs(res - wres) / np.abs(wres)) if wres.size else 0.0
            print(f"D={D} H={H} W={W} sweeps={sweeps}: grid bit-exact={same} residual max rel err={rel:.3g}",
                  flush=True)
            ok = ok and same and rel <= 1e-12
    # Reductions and axpy split across the ranks (one exchange for the sums).
    sh = spmd_mod("shard")
    n = (1 << 22) + 5
    x = np.random.RandomState(0).random_sample(n).astype(np.float32)
    lo, hi = sh.shard_range(n, dist.get_world_size(), rank)
    xl = torch.from_numpy(x[lo:hi]).cuda()
    s1, s2 = sh.sum_f32(xl, init=0.5), sh.sum_f32(xl, init=0.5)
    v = np.random.RandomState(1).randint(0, 100, size=n).astype(np.int32)
    si = sh.sum_i32(torch.from_numpy(v[lo:hi]).cuda(), init=-7)
    y = np.random.RandomState(2).random_sample(n).astype(np.float32)
    yl = torch.from_numpy(y[lo:hi]).cuda()
    sh.axpy(2.5, xl, yl)
    mine = yl.cpu().numpy()
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, (float(s1), int(si)))
    if rank == 0:
        from oracle import oracle
        exact = 0.5 + oracle.sum_f64(x)
        same_all = all(p_ == parts[0] for p_ in parts)
        ok_sum = abs(float(s1) - exact) <= 1e-6 * abs(exact) and s1 == s2 and same_all
        ok_i32 = si == int(v.astype(np.int64).sum()) - 7
        print(f"sharded sums: f32 rel err {abs(float(s1) - exact) / exact:.3g} deterministic={s1 == s2} "
              f"same on every rank={same_all} i32 exact={ok_i32}", flush=True)
        ok = ok and ok_sum and ok_i32
    want_y = None
    if True:
        from oracle import oracle
        want_y = oracle.axpy(2.5, x[lo:hi], y[lo:hi])
    ok_axpy = np.array_equal(mine.view(np.uint32), want_y.view(np.uint32))
    flag_axpy = torch.tensor([1 if ok_axpy else 0], device="cuda")
    dist.all_reduce(flag_axpy, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"sharded axpy bit-exact on every rank={bool(flag_axpy.item())}", flush=True)
        ok = ok and bool(flag_axpy.item())
    # Back-to-back launches with no host synchronisation between them: each
    # kernel waits on the neighbours' monotonic delivery counters (this run's
    # input rows come first), so a rank may start its next run while a
    # neighbour's previous one is still delivering.  Host-buffer runs, which
    # overwrite the slab, wait for every rank's previous launch first.
    G, W = 2048, 4096
    u0 = jacobi_init((G, W), 5)
    job = slab.SlabJacobi2D(cols=W, G=G, res_every=0, init=u0)
    for _ in range(4):
        job.run(9, check=False)
    job.check()
    grid = job.gather()
    host_ok = True
    lo, hi = job.g_first - job.halo, job.g_first + job.rows + job.halo
    from oracle import oracle as orc
    want6, _ = orc.jacobi2d(u0, 6, 0)
    for _ in range(2):  # fresh input each call, as the end-to-end benchmark does
        local = np.zeros((job.local_rows,) + job.unit_shape, np.float32)
        s_lo, s_hi = max(lo, 0), min(hi, G)
        local[s_lo - lo:s_hi - lo] = job._pad(u0[s_lo:s_hi])
        host = torch.empty(local.shape, dtype=torch.float32, pin_memory=True).numpy()
        host[...] = local
        job.run_host(host, 6)
        got = job._trim(host[job.halo:job.halo + job.rows])
        mine6 = want6[job.g_first:job.g_first + job.rows]
        host_ok = host_ok and np.array_equal(got.view(np.uint32), mine6.view(np.uint32))
    job.close()
    flag_host = torch.tensor([1 if host_ok else 0], device="cuda")
    dist.all_reduce(flag_host, op=dist.ReduceOp.MIN)
    if rank == 0:
        want36, _ = orc.jacobi2d(u0, 36, 0)
        same = np.array_equal(grid.view(np.uint32), want36.view(np.uint32))
        print(f"4 back-to-back runs of 9 sweeps: bit-exact={same}; two host-buffer runs: bit-exact="
              f"{bool(flag_host.item())}", flush=True)
        ok = ok and same and bool(flag_host.item())
    # Checkpoint from every rank, resume in a fresh job.
    import tempfile
    ck_dir = tempfile.mkdtemp() if rank == 0 else None
    holder = [ck_dir]
    dist.broadcast_object_list(holder, src=0)
    path = os.path.join(holder[0], "slab.ckpt")
    G, W = 300, 260
    u0 = jacobi_init((G, W), 4)
    a = slab.SlabJacobi2D(cols=W, G=G, res_every=0, init=u0)
    a.run(5)
    a.save(path)
    a.close()
    b = slab.SlabJacobi2D(cols=W, G=G, res_every=0, seed=7)
    b.restore(path)
    b.run(8)
    grid = b.gather()
    b.close()
    if rank == 0:
        from oracle import oracle
        ck = spmd_mod("checkpoint")
        saved, info = ck.load_grid(path)
        mid, _ = oracle.jacobi2d(u0, 5, 0)
        want, _ = oracle.jacobi2d(u0, 13, 0)
        same = (info.sweeps == 5 and np.array_equal(saved.view(np.uint32), mid.view(np.uint32))
                and np.array_equal(grid.view(np.uint32), want.view(np.uint32)))
        print(f"checkpoint from {dist.get_world_size()} ranks, resume: bit-exact={same}", flush=True)
        ok = ok and same
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and bool(flag.item()):
        print("SLAB PARITY OK", flush=True)
    sys.exit(0 if bool(flag.item()) else 1)


if __name__ == "__main__":
    main()
