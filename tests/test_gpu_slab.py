"""Row-slab Jacobi-2D on the GPU.

* one rank (no neighbours) through SlabJacobi2D equals the oracle;
* a bounded peer wait that nothing satisfies (a neighbour whose delivery
  counter is never bumped) ends the kernel with SPMDB200_ERR_TIMEOUT, and the
  context stays usable for the next launch;
* the same for Jacobi-3D z-slabs (one rank; a fake neighbour below);
* with >= 2 GPUs, 2 ranks (torchrun, NCCL plumbing, NVLink halo stores inside
  the kernel) reproduce the single-domain oracle bit for bit, for row slabs
  and z-slabs."""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, assert_bits_equal, jacobi_init, spmd_mod

pytestmark = pytest.mark.gpu


def test_single_rank_slab_matches_oracle(kernels, oracle_mod):
    slab = spmd_mod("slab")
    u0 = jacobi_init((130, 300), 4)
    job = slab.SlabJacobi2D(cols=300, G=130, res_every=2, init=u0)
    job.run(7)
    res = job.residuals()
    got = job.gather()
    job.close()
    want, wres = oracle_mod.jacobi2d(u0, 7, 2)
    assert_bits_equal(got, want, "slab world=1")
    np.testing.assert_allclose(res, wres, rtol=1e-12)


def test_single_rank_seeded_fill_is_deterministic(kernels):
    slab = spmd_mod("slab")
    a = slab.SlabJacobi2D(cols=257, G=65, seed=4)
    b = slab.SlabJacobi2D(cols=257, G=65, seed=4)
    ga, gb = a.gather(), b.gather()
    a.close()
    b.close()
    assert_bits_equal(ga, gb)
    assert ga[0].max() == 0 and ga[-1].max() == 0 and ga[:, 0].max() == 0 and ga[:, -1].max() == 0
    assert 0.4 < float(ga[1:-1, 1:-1].mean()) < 0.6


def test_single_rank_zslab_matches_oracle(kernels, oracle_mod):
    slab = spmd_mod("slab")
    u0 = jacobi_init((21, 40, 300), 3)
    job = slab.SlabJacobi3D(H=40, W=300, D=21, res_every=3, init=u0)
    job.run(7)
    res = job.residuals()
    got = job.gather()
    job.close()
    want, wres = oracle_mod.jacobi3d(u0, 7, 3)
    assert_bits_equal(got, want, "z-slab world=1")
    np.testing.assert_allclose(res, wres, rtol=1e-12)


def test_checkpoint_resume_matches_uninterrupted(kernels, oracle_mod, tmp_path):
    """Run 7 sweeps, save, resume in a fresh job (other seed), run 6: equals 13."""
    slab = spmd_mod("slab")
    u0 = jacobi_init((130, 300), 4)
    a = slab.SlabJacobi2D(cols=300, G=130, res_every=0, init=u0)
    a.run(7)
    a.save(str(tmp_path / "j2.ckpt"))
    a.close()
    b = slab.SlabJacobi2D(cols=300, G=130, res_every=0, seed=99)
    b.restore(str(tmp_path / "j2.ckpt"))
    assert b.sweeps_done == 7
    b.run(6)
    got = b.gather()
    b.close()
    want, _ = oracle_mod.jacobi2d(u0, 13, 0)
    assert_bits_equal(got, want, "2-D resume")
    u3 = jacobi_init((13, 20, 150), 3)
    c = slab.SlabJacobi3D(H=20, W=150, D=13, res_every=0, init=u3)
    c.run(3)
    c.save(str(tmp_path / "j3.ckpt"))
    c.close()
    d = slab.SlabJacobi3D(H=20, W=150, D=13, res_every=0, seed=5)
    d.restore(str(tmp_path / "j3.ckpt"))
    d.run(4)
    got3 = d.gather()
    d.close()
    want3, _ = oracle_mod.jacobi3d(u3, 7, 0)
    assert_bits_equal(got3, want3, "3-D resume")


def test_zslab_seeded_fill_is_deterministic(kernels):
    slab = spmd_mod("slab")
    a = slab.SlabJacobi3D(H=17, W=33, D=9, seed=3)
    b = slab.SlabJacobi3D(H=17, W=33, D=9, seed=3)
    ga, gb = a.gather(), b.gather()
    a.close()
    b.close()
    assert_bits_equal(ga, gb)
    assert ga[0].max() == 0 and ga[-1].max() == 0 and ga[:, 0].max() == 0 and ga[:, :, -1].max() == 0
    assert 0.4 < float(ga[1:-1, 1:-1, 1:-1].mean()) < 0.6


def test_peer_wait_runs_out_and_reports_timeout(kernels):
    """A fake neighbour above (local buffers) whose deliveries never arrive."""
    import torch
    L = spmd_mod("_lib")
    lib = L.lib()
    c_i, c_p = ctypes.c_int64, ctypes.c_void_p
    rows, cols = 64, 256
    H = spmd_mod("slab").HALO
    u = torch.zeros((rows + 2 * H, cols), device="cuda")
    v = torch.zeros_like(u)
    fake_u, fake_v = torch.zeros_like(u), torch.zeros_like(u)
    nbytes = int(lib.spmdb200_jacobi_workspace_bytes())
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    fake_ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")

    def d(t):
        p = c_p(t.data_ptr())
        return (p, p, c_i(0), c_i(rows + 2 * H), c_i(cols), c_i(cols), c_i(1))

    s = c_p(torch.cuda.current_stream().cuda_stream)
    assert lib.spmdb200_set_wait_budget_ms(c_i(2000), c_i(300)) == 0
    try:
        assert lib.spmdb200_jacobi_ws_reset(c_p(ws.data_ptr()), s) == 0
        # this rank owns global rows [64, 128) of 128: a neighbour above, none below
        st = lib.spmdb200_jacobi2d_slab(*d(u), *d(v), c_i(rows), c_i(2 * rows), c_i(3), c_i(0), None,
                                        c_p(ws.data_ptr()), c_p(fake_u.data_ptr()), c_p(fake_v.data_ptr()),
                                        c_p(fake_ws.data_ptr()), c_i(rows), None, None, None, ctypes.c_int(1),
                                        ctypes.c_int(2), (c_p * 2)(c_p(fake_ws.data_ptr()), c_p(ws.data_ptr())),
                                        ctypes.byref(ctypes.c_int64(0)), s)
        assert st == 0, lib.spmdb200_last_error_message()
        st = lib.spmdb200_workspace_status(c_p(ws.data_ptr()), s)
        assert st == -3, "the unsatisfiable peer wait must end in SPMDB200_ERR_TIMEOUT"
        assert b"peer" in lib.spmdb200_last_error_message()
    finally:
        assert lib.spmdb200_set_wait_budget_ms(c_i(4000), c_i(20000)) == 0
    # The context survived: a normal run still works.
    a = torch.rand((64, 128), device="cuda")
    fin, _ = kernels.jacobi2d(a, torch.empty_like(a), 2, 0)
    torch.cuda.synchronize()


def test_zslab_peer_wait_runs_out_and_reports_timeout(kernels):
    """Jacobi-3D: a fake neighbour below (local buffers) that never delivers."""
    import torch
    L = spmd_mod("_lib")
    lib = L.lib()
    c_i, c_p = ctypes.c_int64, ctypes.c_void_p
    planes, H, W = 6, 16, 128
    halo = spmd_mod("slab").HALO3
    u = torch.zeros((planes + 2 * halo, H, W), device="cuda")
    v = torch.zeros_like(u)
    fake_u, fake_v = torch.zeros_like(u), torch.zeros_like(u)
    nbytes = int(lib.spmdb200_jacobi_workspace_bytes())
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    fake_ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")

    def d(t):
        p = c_p(t.data_ptr())
        return (p, p, c_i(0), c_i(planes + 2 * halo), c_i(H), c_i(W), c_i(H * W), c_i(W), c_i(1))

    s = c_p(torch.cuda.current_stream().cuda_stream)
    assert lib.spmdb200_set_wait_budget_ms(c_i(2000), c_i(300)) == 0
    try:
        assert lib.spmdb200_jacobi_ws_reset(c_p(ws.data_ptr()), s) == 0
        # this rank owns global planes [0, 6) of 12: a neighbour below, none above
        st = lib.spmdb200_jacobi3d_slab(*d(u), *d(v), c_i(0), c_i(2 * planes), c_i(3), c_i(0), None,
                                        c_p(ws.data_ptr()), None, None, None, c_i(0),
                                        c_p(fake_u.data_ptr()), c_p(fake_v.data_ptr()), c_p(fake_ws.data_ptr()),
                                        ctypes.c_int(0), ctypes.c_int(2),
                                        (c_p * 2)(c_p(ws.data_ptr()), c_p(fake_ws.data_ptr())),
                                        ctypes.byref(ctypes.c_int64(0)), s)
        assert st == 0, lib.spmdb200_last_error_message()
        st = lib.spmdb200_workspace_status(c_p(ws.data_ptr()), s)
        assert st == -3, "the unsatisfiable peer wait must end in SPMDB200_ERR_TIMEOUT"
        assert b"peer" in lib.spmdb200_last_error_message()
    finally:
        assert lib.spmdb200_set_wait_budget_ms(c_i(4000), c_i(20000)) == 0
    a = torch.rand((8, 16, 128), device="cuda")
    kernels.jacobi3d(a, torch.empty_like(a), 2, 0)
    torch.cuda.synchronize()


def test_two_ranks_match_oracle():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={29600 + os.getpid() % 1000}",
           str(ROOT / "tests" / "slab_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "600", *cmd], capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "SLAB PARITY OK" in r.stdout
