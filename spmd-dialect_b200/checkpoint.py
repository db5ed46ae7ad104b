"""Checkpoint / resume of a Jacobi run: the grid plus its sweep count.

File layout (little-endian): a 64-byte header followed by the global grid as
raw row-major float32 with no padding.

    offset  size  field
    0       8     magic b"SPMDCKP1"
    8       4     header version (1)
    12      4     rank of the grid (2 or 3)
    16      24    extents, int64 x 3 (outermost first; unused entries 0)
    40      8     sweeps already applied to the grid (int64)
    48      8     residual interval of the run (int64, informational)
    56      8     reserved (0)

The grid in the file is the state after `sweeps` sweeps, so a run resumed
from it with k more sweeps equals an uninterrupted run of sweeps + k.  Rows
(2-D) or planes (3-D) are contiguous in the file, so every rank of a slab
decomposition reads and writes only its own block -- a run can resume on a
different number of GPUs.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = b"SPMDCKP1"
VERSION = 1
HEADER = 64
_FMT = "<8sii3qqqq"
assert struct.calcsize(_FMT) == HEADER


@dataclass(frozen=True)
class CheckpointInfo:
    shape: tuple
    sweeps: int
    res_every: int


def write_header(path: str, shape: tuple, sweeps: int, res_every: int = 0) -> None:
    """Creates (or truncates) `path` with a header and room for the grid."""
    if len(shape) not in (2, 3) or any(int(n) < 1 for n in shape):
        raise ValueError(f"checkpoint grids are 2-D or 3-D with positive extents, got {shape}")
    ext = list(int(n) for n in shape) + [0] * (3 - len(shape))
    head = struct.pack(_FMT, MAGIC, VERSION, len(shape), *ext, int(sweeps), int(res_every), 0)
    nbytes = HEADER + 4 * int(np.prod(shape))
    with open(path, "wb") as f:
        f.write(head)
        f.truncate(nbytes)


def read_header(path: str) -> CheckpointInfo:
    with open(path, "rb") as f:
        raw = f.read(HEADER)
    if len(raw) != HEADER:
        raise ValueError(f"{path}: truncated checkpoint header")
    magic, version, rank, e0, e1, e2, sweeps, res_every, _ = struct.unpack(_FMT, raw)
    if magic != MAGIC or version != VERSION or rank not in (2, 3):
        raise ValueError(f"{path}: not a checkpoint of this format (magic {magic!r}, version {version})")
    shape = (e0, e1) if rank == 2 else (e0, e1, e2)
    if os.path.getsize(path) != HEADER + 4 * int(np.prod(shape)):
        raise ValueError(f"{path}: size does not match the header's grid {shape}")
    return CheckpointInfo(shape, sweeps, res_every)


def _map(path: str, mode: str) -> np.memmap:
    info = read_header(path)
    return np.memmap(path, dtype=np.float32, mode=mode, offset=HEADER, shape=info.shape)


def write_block(path: str, first: int, block: np.ndarray) -> None:
    """Writes units (rows or planes) [first, first + len(block)) of the grid."""
    m = _map(path, "r+")
    if block.shape[1:] != m.shape[1:] or first < 0 or first + block.shape[0] > m.shape[0]:
        raise ValueError(f"block {block.shape} at {first} does not fit grid {m.shape}")
    m[first:first + block.shape[0]] = block
    m.flush()
    del m


def read_block(path: str, lo: int, hi: int) -> np.ndarray:
    """Units [lo, hi) of the grid; units outside the grid read as 0."""
    m = _map(path, "r")
    out = np.zeros((hi - lo,) + m.shape[1:], np.float32)
    a, b = max(lo, 0), min(hi, m.shape[0])
    if b > a:
        out[a - lo:b - lo] = m[a:b]
    del m
    return out


def save_grid(path: str, grid: np.ndarray, sweeps: int, res_every: int = 0) -> None:
    """One-process save of a whole grid (host array)."""
    write_header(path, grid.shape, sweeps, res_every)
    write_block(path, 0, np.ascontiguousarray(grid, np.float32))


def load_grid(path: str) -> tuple[np.ndarray, CheckpointInfo]:
    info = read_header(path)
    return read_block(path, 0, info.shape[0]), info


def save_tensor(path: str, grid, sweeps: int, res_every: int = 0) -> None:
    """Saves a device (or host) torch tensor holding the current grid."""
    save_grid(path, grid.detach().to("cpu").contiguous().numpy(), sweeps, res_every)


def load_tensor(path: str, device="cuda"):
    """(grid tensor on `device`, info) from a checkpoint."""
    import torch
    grid, info = load_grid(path)
    return torch.from_numpy(grid).to(device), info
