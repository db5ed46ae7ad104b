"""Shared fixtures.  `-m gpu` tests need a CUDA device and the built library;
everything else runs on CPU (oracle vs golden fixtures, ABI checks, host logic,
gloo multi-rank tests)."""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libspmdb200.so")


def spmd_pkg():
    """The product package (directory name has a hyphen, so importlib)."""
    return importlib.import_module("spmd-dialect_b200")


def spmd_mod(name: str):
    return importlib.import_module(f"spmd-dialect_b200.{name}")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def kernels():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return spmd_mod("kernels")


@pytest.fixture(scope="session")
def host_api():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return spmd_mod("host")


def jacobi_init(shape, seed: int) -> np.ndarray:
    """Interior uniform [0,1) from RandomState(seed), boundary cells 0."""
    rng = np.random.RandomState(seed)
    u = rng.random_sample(shape).astype(np.float32)
    if u.ndim == 2:
        u[0, :] = 0; u[-1, :] = 0; u[:, 0] = 0; u[:, -1] = 0
    else:
        u[0] = 0; u[-1] = 0; u[:, 0] = 0; u[:, -1] = 0; u[:, :, 0] = 0; u[:, :, -1] = 0
    return u


def assert_bits_equal(a: np.ndarray, b: np.ndarray, what: str = "") -> None:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    av, bv = a.view(np.uint32), b.view(np.uint32)
    bad = np.nonzero(av != bv)
    if bad[0].size:
        idx = tuple(x[0] for x in bad)
        raise AssertionError(f"{what}: {bad[0].size} cells differ; first at {idx}: {a[idx]!r} vs {b[idx]!r}")
