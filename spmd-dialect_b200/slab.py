"""Slab decompositions across GPUs: row slabs for Jacobi-2D, plane (z) slabs
for Jacobi-3D.  One process per GPU.

torch.distributed is plumbing only (exchanging CUDA IPC handles, the
rendezvous around host-side reads and writes of the slabs, gathering results
for tests).  The data path --
the halo exchange and the residual all-gather every `res_every` sweeps -- runs
inside the persistent kernels over NVLink (spmdb200_jacobi2d_slab,
spmdb200_jacobi3d_slab): no NCCL call sits between sweeps.

Jacobi-2D: the G x W global grid is cut into contiguous row blocks; rank p owns
global rows [g_first, g_first + rows) and keeps a (rows + 16) x pitch local
array whose first and last HALO = 8 rows mirror the neighbours' edge rows
(eight rows deep, because the kernel fuses up to eight sweeps per pass; eight
rows move up and eight down per pass, and each run first sends the edge rows
of its input).

The kernels wait on halo-delivery counters that only grow; each job keeps
the count it has received so far and passes it to every run, so runs follow
one another with no host synchronisation between them.

Jacobi-3D: the D x H x W grid is cut into contiguous plane blocks; rank p owns
planes [g_first, g_first + planes) plus HALO3 = 2 halo planes on each side (up
to two sweeps per pass, two planes up and two down per pass; each run first
sends the edge planes of its input).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import c_i, c_p, call, lib

HALO = int(lib().spmdb200_jacobi_slab_halo(2))  # halo rows on each side of a 2-D slab (8)
HALO3 = int(lib().spmdb200_jacobi_slab_halo(3))  # halo planes on each side of a 3-D slab (2)


# ---------------------------------------------------------------- decomposition
def partition(G: int, world: int, rank: int) -> tuple[int, int]:
    """(g_first, rows) of `rank`'s contiguous block of the G global rows."""
    if not (0 <= rank < world) or G < world:
        raise ValueError(f"cannot split {G} rows over {world} ranks")
    base, extra = divmod(G, world)
    rows = base + (1 if rank < extra else 0)
    return rank * base + min(rank, extra), rows


def neighbours(G: int, world: int, rank: int) -> tuple[int | None, int | None]:
    """Ranks owning the rows just above and just below this rank's block."""
    return (rank - 1 if rank > 0 else None), (rank + 1 if rank < world - 1 else None)


def local_row_range(G: int, world: int, rank: int, halo: int = HALO) -> tuple[int, int]:
    """Global rows [lo, hi) a rank's local array mirrors: its block plus `halo`
    rows on each side (rows outside [0, G) exist locally but are never read)."""
    g_first, rows = partition(G, world, rank)
    return g_first - halo, g_first + rows + halo


def pitch_for(cols: int) -> int:
    """Row pitch in floats: a multiple of 4 so every row is 16-byte aligned (TMA)."""
    return (cols + 3) & ~3


# ---------------------------------------------------------------- device memory
class DeviceBuffer:
    """cudaMalloc'd device memory (IPC-shareable), freed by close()."""

    def __init__(self, nbytes: int):
        p = c_p()
        call("spmdb200_dev_alloc", ctypes.c_size_t(nbytes), ctypes.byref(p))
        self.ptr = p.value
        self.nbytes = nbytes

    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        call("spmdb200_ipc_handle", c_p(self.ptr), buf)
        return buf.raw

    def close(self) -> None:
        if self.ptr:
            call("spmdb200_dev_free", c_p(self.ptr))
            self.ptr = 0


def ipc_open(handle: bytes) -> int:
    p = c_p()
    call("spmdb200_ipc_open", ctypes.create_string_buffer(handle, 64), ctypes.byref(p))
    return p.value


@dataclass
class _Peer:
    u: int = 0
    v: int = 0
    ws: int = 0


def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() else None


def rendezvous() -> None:
    """Every rank reaches this point before any rank goes on (job set-up, host
    reads and writes of the slabs, close): a rank that never arrives makes the
    others fail here with the process-group timeout."""
    d = _dist()
    if d is not None and d.get_world_size() > 1:
        d.barrier()


class _SlabJob:
    """Plumbing shared by the row-slab (2-D) and plane-slab (3-D) jobs: the split
    axis holds `G` global units (rows or planes); this rank owns `rows` of them
    from `g_first` and keeps `local_rows = rows + 2 * halo` units locally, each
    `unit_shape` floats (a padded row, or a plane of padded rows)."""

    halo: int
    entry: str
    unit_shape: tuple

    def _setup(self, G: int, res_every: int, seed: int, init: np.ndarray | None) -> None:
        import torch
        d = _dist()
        self.rank = d.get_rank() if d else 0
        self.world = d.get_world_size() if d else 1
        self.G, self.res_every = G, res_every
        self.g_first, self.rows = partition(G, self.world, self.rank)
        if self.rows < self.halo:
            raise ValueError(f"each rank needs >= {self.halo} units (rank {self.rank} has {self.rows})")
        self.local_rows = self.rows + 2 * self.halo
        self.unit_floats = int(np.prod(self.unit_shape))
        nbytes = self.local_rows * self.unit_floats * 4
        self._u = DeviceBuffer(nbytes)
        self._v = DeviceBuffer(nbytes)
        self._ws = DeviceBuffer(int(lib().spmdb200_jacobi_workspace_bytes()))
        self.sweeps_done = 0
        self._nres_last = 0
        self._deliveries = ctypes.c_int64(0)  # halo deliveries received from each neighbour so far
        stream = c_p(torch.cuda.current_stream().cuda_stream)
        call("spmdb200_jacobi_ws_reset", c_p(self._ws.ptr), stream)
        if init is None:
            for buf in (self._u, self._v):
                self._fill(buf.ptr, seed, stream)
        else:
            self.load_global(init)
        # Every workspace is clear before the handle exchange below, which no
        # rank passes before all have arrived: no kernel can deliver into an
        # uncleared workspace.
        torch.cuda.current_stream().synchronize()
        # Map the neighbours' grids and every rank's workspace into this process.
        self._up, self._dn = _Peer(), _Peer()
        self._up_rows = 0
        self._all_ws = [0] * self.world
        self._opened: list[int] = []
        self._all_ws[self.rank] = self._ws.ptr
        if self.world > 1:
            mine = (self._u.ipc_handle(), self._v.ipc_handle(), self._ws.ipc_handle())
            handles: list = [None] * self.world
            d.all_gather_object(handles, mine)
            up, dn = neighbours(G, self.world, self.rank)
            if up is not None:
                self._up_rows = partition(G, self.world, up)[1]
            for q in range(self.world):
                if q != self.rank:
                    self._all_ws[q] = self._open(handles[q][2])
            if up is not None:
                self._up = _Peer(self._open(handles[up][0]), self._open(handles[up][1]), self._all_ws[up])
            if dn is not None:
                self._dn = _Peer(self._open(handles[dn][0]), self._open(handles[dn][1]), self._all_ws[dn])
        self._all_ws_arr = (c_p * max(self.world, 1))(*[c_p(x) for x in self._all_ws])

    def _open(self, h: bytes) -> int:
        p = ipc_open(h)
        self._opened.append(p)
        return p

    # ---------------------------------------------------------------- data movement
    def _trim(self, local: np.ndarray) -> np.ndarray:
        """Owned units of a host copy of the local array, padding columns removed."""
        raise NotImplementedError

    def _pad(self, block: np.ndarray) -> np.ndarray:
        """Global units (unpadded) -> the local layout's padded units."""
        raise NotImplementedError

    def load_global(self, grid: np.ndarray) -> None:
        """Copies this rank's units (+ halos) of the global grid into U (and V)."""
        lo, hi = self.g_first - self.halo, self.g_first + self.rows + self.halo
        local = np.zeros((self.local_rows,) + self.unit_shape, np.float32)
        src_lo, src_hi = max(lo, 0), min(hi, self.G)
        local[src_lo - lo:src_hi - lo] = self._pad(np.asarray(grid[src_lo:src_hi], np.float32))
        for buf in (self._u, self._v):
            call("spmdb200_memcpy", c_p(buf.ptr), local.ctypes.data_as(c_p), ctypes.c_size_t(local.nbytes), None)
        self.sweeps_done = 0

    def local_owned(self) -> np.ndarray:
        """This rank's owned units of the current grid (host copy)."""
        local = np.empty((self.local_rows,) + self.unit_shape, np.float32)
        call("spmdb200_memcpy", local.ctypes.data_as(c_p), c_p(self._u.ptr), ctypes.c_size_t(local.nbytes), None)
        return self._trim(local[self.halo:self.halo + self.rows])

    def gather(self) -> np.ndarray | None:
        """The full global grid on rank 0 (None elsewhere)."""
        mine = self.local_owned()
        d = _dist()
        if d is None or self.world == 1:
            return mine
        parts: list = [None] * self.world if self.rank == 0 else None
        d.gather_object(mine, parts, dst=0)
        return np.concatenate(parts, axis=0) if self.rank == 0 else None

    # ---------------------------------------------------------------- checkpoint / resume
    def save(self, path: str) -> None:
        """Checkpoint: rank 0 writes the header, then every rank writes its owned
        units of the current grid at their offset (collective: all ranks call)."""
        from . import checkpoint as ck
        if self.rank == 0:
            ck.write_header(path, (self.G,) + self._global_unit_shape(), self.sweeps_done, self.res_every)
        rendezvous()
        ck.write_block(path, self.g_first, self.local_owned())
        rendezvous()

    def restore(self, path: str) -> None:
        """Loads this rank's units (+ halos) of a checkpointed grid into U and V and
        takes over its sweep count.  The checkpoint may come from any number of ranks."""
        from . import checkpoint as ck
        info = ck.read_header(path)
        want = (self.G,) + self._global_unit_shape()
        if tuple(info.shape) != want:
            raise ValueError(f"checkpoint grid {info.shape} does not match this job's grid {want}")
        block = ck.read_block(path, self.g_first - self.halo, self.g_first + self.rows + self.halo)
        local = np.ascontiguousarray(self._pad(block))
        self._quiesce()
        for buf in (self._u, self._v):
            call("spmdb200_memcpy", c_p(buf.ptr), local.ctypes.data_as(c_p), ctypes.c_size_t(local.nbytes), None)
        self.sweeps_done = info.sweeps
        rendezvous()

    # ---------------------------------------------------------------- running
    def _quiesce(self) -> None:
        """Returns once every rank's previous launch is complete.  A launch's
        last pass still stores halo rows into the neighbours' memory after a
        neighbour's own kernel may have ended; host code that overwrites a
        slab (a load or a restore) must not race with those stores."""
        import torch
        torch.cuda.current_stream().synchronize()
        rendezvous()

    def run(self, sweeps: int, check: bool = True) -> None:
        """`sweeps` sweeps on every rank (all ranks must call with the same
        count).  Asynchronous on the current stream: the kernel itself waits
        for the neighbours' halo rows, so no host synchronisation comes first."""
        import torch
        stream = c_p(torch.cuda.current_stream().cuda_stream)
        up, dn = self._up, self._dn
        call(self.entry, *self._desc(self._u.ptr), *self._desc(self._v.ptr), c_i(self.g_first),
             c_i(self.G), c_i(sweeps), c_i(self.res_every), c_p(0), c_p(self._ws.ptr),
             c_p(up.u or None), c_p(up.v or None), c_p(up.ws or None), c_i(self._up_rows),
             c_p(dn.u or None), c_p(dn.v or None), c_p(dn.ws or None),
             ctypes.c_int(self.rank), ctypes.c_int(self.world), self._all_ws_arr, ctypes.byref(self._deliveries),
             stream)
        self._nres_last = sweeps // self.res_every if self.res_every > 0 else 0
        self.sweeps_done += sweeps
        if sweeps % 2 == 1:
            # The result sits in V on every rank: swap roles so U is current everywhere.
            self._u, self._v = self._v, self._u
            up.u, up.v = up.v, up.u
            dn.u, dn.v = dn.v, dn.u
        if check:
            self.check()

    def check(self) -> None:
        """Synchronises and raises SpmdError if this rank's kernel hit a bounded-wait timeout."""
        import torch
        call("spmdb200_workspace_status", c_p(self._ws.ptr), c_p(torch.cuda.current_stream().cuda_stream))

    def residuals(self) -> np.ndarray:
        """Global residuals (sum of squared updates) of the last run, identical on every rank."""
        import torch
        torch.cuda.current_stream().synchronize()
        rendezvous()  # every rank's kernel has finished writing its slots
        out = np.zeros(max(self._nres_last, 1), np.float64)
        call("spmdb200_jacobi2d_slab_residuals", c_p(self._ws.ptr), ctypes.c_int(self.world),
             c_i(self._nres_last), out.ctypes.data_as(c_p))
        rendezvous()  # no rank's next run writes the slots before every rank has read them
        return out[:self._nres_last]

    def run_host(self, host_local: np.ndarray, sweeps: int) -> np.ndarray:
        """End to end on host memory: host_local is this rank's local array
        (local_rows x unit_shape, pinned for full speed); copied in, `sweeps`
        sweeps, owned units copied back into host_local[halo:halo + rows]."""
        if host_local.shape != (self.local_rows,) + self.unit_shape or host_local.dtype != np.float32:
            raise ValueError(f"host slab must be {(self.local_rows,) + self.unit_shape} float32")
        # Only U needs the input: V's owned units are all written by the first
        # sweep and its halo units by the neighbours before anyone reads them.
        self._quiesce()
        call("spmdb200_memcpy", c_p(self._u.ptr), host_local.ctypes.data_as(c_p),
             ctypes.c_size_t(host_local.nbytes), None)
        self.run(sweeps, check=True)
        unit = self.unit_floats * 4
        call("spmdb200_memcpy", c_p(host_local.ctypes.data + self.halo * unit), c_p(self._u.ptr + self.halo * unit),
             ctypes.c_size_t(self.rows * unit), None)
        return host_local

    def close(self) -> None:
        import torch
        torch.cuda.synchronize()
        rendezvous()  # no peer still writes into our memory or reads our workspace
        for p in self._opened:
            call("spmdb200_ipc_close", c_p(p))
        self._opened = []
        rendezvous()
        for b in (self._u, self._v, self._ws):
            b.close()


class SlabJacobi2D(_SlabJob):
    """This rank's share of a multi-GPU Jacobi-2D run (row slabs, spmdb200_jacobi2d_slab).

    G x cols global grid (G defaults to rows_per_rank * world: weak scaling).
    `init` is None (seeded synthetic input generated on the device, identical
    to what a single-GPU run of the same global grid would see) or the full
    global grid as a numpy array (tests)."""

    halo = HALO
    entry = "spmdb200_jacobi2d_slab"

    def __init__(self, cols: int, rows_per_rank: int | None = None, G: int | None = None, seed: int = 4,
                 res_every: int = 10, init: np.ndarray | None = None):
        d = _dist()
        world = d.get_world_size() if d else 1
        if G is None:
            if rows_per_rank is None:
                raise ValueError("give rows_per_rank or G")
            G = rows_per_rank * world
        self.cols = cols
        self.pitch = pitch_for(cols)
        self.unit_shape = (self.pitch,)
        self._setup(G, res_every, seed, init)

    def _global_unit_shape(self) -> tuple:
        return (self.cols,)

    def twin(self) -> "SlabJacobi2D":
        """A job with the same decomposition (a second device slot)."""
        return SlabJacobi2D(cols=self.cols, G=self.G, seed=4, res_every=self.res_every)

    def _fill(self, ptr: int, seed: int, stream) -> None:
        call("spmdb200_fill_jacobi_input", c_p(ptr), c_i(self.pitch), c_i(self.local_rows), c_i(self.cols),
             c_i(self.g_first - self.halo), c_i(self.G), ctypes.c_uint64(seed), stream)

    def _desc(self, ptr: int) -> tuple:
        p = c_p(ptr)
        return (p, p, c_i(0), c_i(self.local_rows), c_i(self.cols), c_i(self.pitch), c_i(1))

    def _trim(self, local: np.ndarray) -> np.ndarray:
        return local[:, :self.cols].copy()

    def _pad(self, block: np.ndarray) -> np.ndarray:
        out = np.zeros((block.shape[0], self.pitch), np.float32)
        out[:, :self.cols] = block
        return out


class SlabJacobi3D(_SlabJob):
    """This rank's share of a multi-GPU Jacobi-3D run (z-slabs,
    spmdb200_jacobi3d_slab): D x H x W global grid split into contiguous plane
    blocks, two halo planes on each side (HALO3).  Same API as SlabJacobi2D."""

    halo = HALO3
    entry = "spmdb200_jacobi3d_slab"

    def __init__(self, H: int, W: int, planes_per_rank: int | None = None, D: int | None = None, seed: int = 3,
                 res_every: int = 10, init: np.ndarray | None = None):
        d = _dist()
        world = d.get_world_size() if d else 1
        if D is None:
            if planes_per_rank is None:
                raise ValueError("give planes_per_rank or D")
            D = planes_per_rank * world
        self.H, self.cols = H, W
        self.pitch = pitch_for(W)
        self.unit_shape = (H, self.pitch)
        self._setup(D, res_every, seed, init)

    @property
    def planes(self) -> int:
        return self.rows

    def _global_unit_shape(self) -> tuple:
        return (self.H, self.cols)

    def twin(self) -> "SlabJacobi3D":
        """A job with the same decomposition (a second device slot)."""
        return SlabJacobi3D(H=self.H, W=self.cols, D=self.G, seed=3, res_every=self.res_every)

    def _fill(self, ptr: int, seed: int, stream) -> None:
        call("spmdb200_fill_jacobi3d_input", c_p(ptr), c_i(self.H * self.pitch), c_i(self.pitch),
             c_i(self.local_rows), c_i(self.H), c_i(self.cols), c_i(self.g_first - self.halo), c_i(self.G),
             ctypes.c_uint64(seed), stream)

    def _desc(self, ptr: int) -> tuple:
        p = c_p(ptr)
        return (p, p, c_i(0), c_i(self.local_rows), c_i(self.H), c_i(self.cols), c_i(self.H * self.pitch),
                c_i(self.pitch), c_i(1))

    def _trim(self, local: np.ndarray) -> np.ndarray:
        return local[:, :, :self.cols].copy()

    def _pad(self, block: np.ndarray) -> np.ndarray:
        out = np.zeros((block.shape[0], self.H, self.pitch), np.float32)
        out[:, :, :self.cols] = block
        return out


def run_host_pipelined(jobs: list, hosts: list, sweeps: int, steps: int) -> None:
    """`steps` runs of `sweeps` sweeps on host slabs, pipelined across two
    device slots.  jobs: two slab jobs (SlabJacobi2D or SlabJacobi3D) with the
    same decomposition (the slots); hosts: two pinned host arrays of this
    rank's owned rows or planes, used alternately -- run k reads
    hosts[k % 2] and writes its result back there.  Uploads, sweeps and downloads run on three
    streams, so run k's sweeps overlap the download of run k-1 and the upload
    of run k+1 (which waits for that download: they share a host buffer).
    Only owned rows / planes cross PCIe: every run first delivers its input's
    edge rows / planes into the neighbours' halos itself.  All ranks call it with the same
    arguments; it returns once every copy of this rank has finished."""
    import torch
    if (len(jobs) != 2 or len(hosts) != 2 or type(jobs[0]) is not type(jobs[1])
            or not isinstance(jobs[0], (SlabJacobi2D, SlabJacobi3D))):
        raise ValueError("two slab jobs of one kind (slots) and two host arrays are required")
    own = jobs[0].rows * jobs[0].unit_floats * 4
    off = jobs[0].halo * jobs[0].unit_floats * 4
    for h in hosts:
        if h.nbytes != own or not h.flags["C_CONTIGUOUS"]:
            raise ValueError(f"host slabs must be contiguous {own}-byte arrays of the owned rows")
    comp = torch.cuda.current_stream()
    up, dn = torch.cuda.Stream(), torch.cuda.Stream()
    ev_up = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_dn = [torch.cuda.Event() for _ in range(2)]
    for k in range(steps):
        j, h, e = jobs[k % 2], hosts[k % 2], k % 2
        if k >= 2:
            up.wait_event(ev_dn[e])  # the download of run k-2 used this host array and slot
        call("spmdb200_memcpy_async", c_p(j._u.ptr + off), c_p(h.ctypes.data), ctypes.c_size_t(own),
             c_p(up.cuda_stream))
        ev_up[e].record(up)
        comp.wait_event(ev_up[e])
        j.run(sweeps, check=False)
        ev_comp[e].record(comp)
        dn.wait_event(ev_comp[e])
        call("spmdb200_memcpy_async", c_p(h.ctypes.data), c_p(j._u.ptr + off), ctypes.c_size_t(own),
             c_p(dn.cuda_stream))
        ev_dn[e].record(dn)
    for s_ in (up, comp, dn):
        s_.synchronize()
    for j in jobs:
        j.check()


def e2e_measure(job: _SlabJob, sweeps: int, steps: int = 3, reps: int = 2) -> dict:
    """Whole-job end-to-end rate with pinned host slabs, every copy inside the
    timed region, wall clock, max over ranks: `steps` host slabs per rank
    through run_host_pipelined (a twin job is the second device slot)."""
    import time

    import torch
    d = _dist()
    cells = job.G * job.cols * (job.H if isinstance(job, SlabJacobi3D) else 1)
    twin = job.twin()
    hosts = [torch.empty((job.rows,) + job.unit_shape, dtype=torch.float32, pin_memory=True).numpy()
             for _ in range(2)]
    own = job.rows * job.unit_floats * 4
    for h in hosts:  # input: the job's current owned rows / planes
        call("spmdb200_memcpy", c_p(h.ctypes.data), c_p(job._u.ptr + job.halo * job.unit_floats * 4),
             ctypes.c_size_t(own), None)
    run_host_pipelined([job, twin], hosts, 2, 2)  # warm-up: both slots, copies and launches
    rendezvous()
    t0 = time.perf_counter()
    run_host_pipelined([job, twin], hosts, sweeps, steps)
    secs = time.perf_counter() - t0
    twin.close()
    t = torch.tensor([secs], dtype=torch.float64, device="cuda")
    if d is not None and job.world > 1:
        d.all_reduce(t, op=d.ReduceOp.MAX)
    secs = float(t.item())
    unit = "rows" if isinstance(job, SlabJacobi2D) else "planes"
    return {"value": round(steps * cells * sweeps / secs / 1e9, 3), "unit": "Gcell-updates/s",
            "h2d_bytes_per_step": own, "d2h_bytes_per_step": own,
            "entry": f"slab.run_host_pipelined: {steps} pinned host slabs per rank (owned {unit}), two device "
                     "slots, uploads and downloads overlapping the sweeps, wall clock"}
