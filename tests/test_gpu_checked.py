"""The general kernels' parity suites rerun against the checked build
(libspmdb200_checked.so: run-time index checks that record instead of
trapping, shared tiles poisoned with NaN before staging).  Any cell the
staging leaves unwritten but the stencil reads comes out NaN and fails the
bit-exact comparison with the oracle; any out-of-range index is skipped and
recorded, and the record must stay empty."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

SUITES = ["tests/test_gpu_forall_map.py", "tests/test_gpu_stencil_nd.py", "tests/test_gpu_mlir_shim.py"]

CHILD = """
import ctypes, importlib, sys
import pytest
rc = pytest.main(["-q", "-x", "-m", "gpu", "-p", "no:cacheprovider", *sys.argv[1:]])
L = importlib.import_module("spmd-dialect_b200._lib")
v = ctypes.c_uint64(0)
st = L.lib().spmdb200_check_status(ctypes.byref(v))
print("LIBRARY", L.LIB_PATH.name)
print("CHECK_STATUS", st, hex(v.value), L.lib().spmdb200_last_error_message().decode())
sys.exit(int(rc) or (st != 0))
"""


def test_parity_suites_on_the_checked_build(kernels):
    lib = ROOT / "spmd-dialect_b200" / "libspmdb200_checked.so"
    assert lib.exists(), "libspmdb200_checked.so is not built (spmd-dialect_b200/build.py)"
    env = dict(os.environ, SPMDB200_VARIANT="checked")
    r = subprocess.run([sys.executable, "-c", CHILD, *SUITES], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=1200)
    out = r.stdout + r.stderr
    assert "LIBRARY libspmdb200_checked.so" in r.stdout, out[-3000:]
    assert r.returncode == 0 and "CHECK_STATUS 0 0x0" in r.stdout, out[-4000:]
