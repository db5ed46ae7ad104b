"""C-ABI checks that need no GPU: the library loads, exports every function
include/spmd_b200.h declares, the cubin carries the reference kernel names,
bad descriptors are rejected before any CUDA call, and -- on a machine with no
GPU -- a valid call fails loudly instead of falling back to the CPU."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT, spmd_mod

HEADER = ROOT / "include" / "spmd_b200.h"
REF_KERNELS = ["ewise_kernel", "promoted_stencil_kernel", "promoted_stencil_kernel_square",
               "atomic_sum_kernel", "hierarchical_sum_kernel"]


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in {"defined"}))


def test_header_declares_reference_names():
    names = declared_functions()
    for n in ["ewise", "stencil_cpu", "atomic_sum", "hierarchical_sum", "spmdb200_jacobi2d", "spmdb200_sum_f32"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = spmd_mod("_lib").lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_cubin_has_reference_entry_names():
    cubin = spmd_mod("_lib").CUBIN_PATH
    assert cubin.exists(), "spmdb200_kernels.cubin not built"
    out = subprocess.run(["nm", str(cubin)], capture_output=True, text=True)
    syms = out.stdout if out.returncode == 0 else cubin.read_bytes().decode("latin-1")
    for k in REF_KERNELS:
        assert re.search(rf"\b{k}\b", syms), f"{k} missing from the cubin"


def test_version_string():
    assert "sm_100a" in spmd_mod("_lib").lib().spmdb200_version().decode()


def _d1(p, n, stride=1, off=0):
    c_i = ctypes.c_int64
    return (ctypes.c_void_p(p), ctypes.c_void_p(p), c_i(off), c_i(n), c_i(stride))


@pytest.mark.parametrize("case", ["neg_n", "null", "short", "zero_stride", "neg_off"])
def test_bad_descriptor_rejected_before_launch(case):
    L = spmd_mod("_lib")
    lib = L.lib()
    fake = 0x1000  # never dereferenced: validation fails first
    c_i = ctypes.c_int64
    a = _d1(fake, 100)
    n = 100
    if case == "neg_n":
        n = -1
    elif case == "null":
        a = _d1(0, 100)
    elif case == "short":
        a = _d1(fake, 50)
    elif case == "zero_stride":
        a = _d1(fake, 100, stride=0)
    elif case == "neg_off":
        a = _d1(fake, 100, off=-4)
    st = lib.spmdb200_ewise(*a, *_d1(fake, 100), *_d1(fake, 100), c_i(n), None)
    assert st == -1
    assert lib.spmdb200_last_error() == -1
    assert lib.spmdb200_last_error_message()


def test_jacobi_rejects_mismatched_and_bad_workspace():
    lib = spmd_mod("_lib").lib()
    c_i = ctypes.c_int64
    fake = ctypes.c_void_p(0x1000)

    def d2(n0, n1, s0):
        return (fake, fake, c_i(0), c_i(n0), c_i(n1), c_i(s0), c_i(1))

    wsb = lib.spmdb200_jacobi_workspace_bytes()
    assert wsb >= 256
    st = lib.spmdb200_jacobi2d(*d2(8, 8, 8), *d2(8, 9, 9), c_i(1), c_i(0), None, fake, ctypes.c_size_t(wsb), None)
    assert st == -1
    st = lib.spmdb200_jacobi2d(*d2(8, 8, 8), *d2(8, 8, 8), c_i(1), c_i(0), None, None, ctypes.c_size_t(wsb), None)
    assert st == -5
    st = lib.spmdb200_jacobi2d(*d2(8, 8, 8), *d2(8, 8, 8), c_i(4), c_i(2), None, fake, ctypes.c_size_t(wsb), None)
    assert st == -1  # residuals due but no res_out


def test_sum_workspace_contract():
    lib = spmd_mod("_lib").lib()
    c_i = ctypes.c_int64
    need = lib.spmdb200_sum_workspace_bytes(c_i(1 << 24))
    assert need >= 256 + 8
    fake = ctypes.c_void_p(0x1000)
    o = (fake, fake, c_i(0))
    st = lib.spmdb200_sum_f32(*_d1(0x1000, 10), *o, c_i(10), ctypes.c_void_p(0x1010), ctypes.c_size_t(need), None)
    assert st == -5  # misaligned workspace
    st = lib.spmdb200_sum_f32(*_d1(0x1000, 10), *o, c_i(10), fake, ctypes.c_size_t(8), None)
    assert st == -5  # too small


def test_no_silent_cpu_fallback_without_gpu():
    """With no usable GPU a valid host-entry call must report an error, never compute on the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the -m gpu tests")
    import numpy as np
    host = spmd_mod("host")
    a = np.ones(16, np.float32)
    b = np.ones(16, np.float32)
    c = np.zeros(16, np.float32)
    with pytest.raises(spmd_mod("_lib").SpmdError):
        host.ewise(a, b, c)
    assert not c.any(), "output written without a GPU"


def test_jacobi2d_host_batch_validates_and_never_falls_back():
    """The batch host entry checks its arguments before any CUDA call, and with
    no usable GPU reports an error instead of sweeping on the CPU."""
    import numpy as np
    import torch
    lib = spmd_mod("_lib").lib()
    c_i = ctypes.c_int64
    fake = (ctypes.c_void_p * 1)(0x1000)
    grids = ctypes.cast(fake, ctypes.c_void_p)
    assert lib.spmdb200_jacobi2d_host_batch(c_i(-1), grids, c_i(0), c_i(8), c_i(8), c_i(8), c_i(1), c_i(1), c_i(0),
                                            None) == -1
    assert lib.spmdb200_jacobi2d_host_batch(c_i(1), None, c_i(0), c_i(8), c_i(8), c_i(8), c_i(1), c_i(1), c_i(0),
                                            None) == -1
    assert lib.spmdb200_jacobi2d_host_batch(c_i(1), grids, c_i(0), c_i(8), c_i(8), c_i(8), c_i(2), c_i(1), c_i(0),
                                            None) == -4  # rows must be contiguous
    assert lib.spmdb200_jacobi2d_host_batch(c_i(1), grids, c_i(0), c_i(8), c_i(8), c_i(4), c_i(1), c_i(1), c_i(0),
                                            None) == -1  # row pitch below the row length
    assert lib.spmdb200_jacobi2d_host_batch(c_i(1), grids, c_i(0), c_i(8), c_i(8), c_i(8), c_i(1), c_i(4), c_i(2),
                                            None) == -1  # residuals due but nowhere to put them
    if torch.cuda.is_available():
        return
    host = spmd_mod("host")
    gs = [np.ones((6, 8), np.float32) for _ in range(2)]
    with pytest.raises(spmd_mod("_lib").SpmdError):
        host.jacobi2d_host_batch(gs, 3)
    assert all((g == 1).all() for g in gs), "grid changed without a GPU"


def test_jacobi2d_host_batch_wrapper_checks_layout():
    """Every grid of a batch shares one shape and row pitch, rows contiguous."""
    import numpy as np
    host = spmd_mod("host")
    a = np.zeros((6, 8), np.float32)
    assert host.jacobi2d_host_batch([], 3) == []
    for bad in ([a, np.zeros((6, 9), np.float32)],            # shape differs
                [a, np.zeros((6, 16), np.float32)[:, :8]],    # row pitch differs
                [np.zeros((6, 16), np.float32)[:, ::2]],      # rows not contiguous
                [a.astype(np.float64)]):                       # not float32
        with pytest.raises(ValueError):
            host.jacobi2d_host_batch(bad, 3)


def test_check_status_release_and_checked_exports():
    """The release library answers 'not a checked build' without a CUDA call;
    the checked library exports every declared function too."""
    lib = spmd_mod("_lib").lib()
    v = ctypes.c_uint64(1)
    if spmd_mod("_lib").VARIANT != "checked":
        assert lib.spmdb200_check_status(ctypes.byref(v)) == -4 and v.value == 0
    checked = ROOT / "spmd-dialect_b200" / "libspmdb200_checked.so"
    assert checked.exists(), "libspmdb200_checked.so not built"
    ch = ctypes.CDLL(str(checked))
    missing = [n for n in declared_functions() if not hasattr(ch, n)]
    assert not missing, f"not exported by the checked build: {missing}"


C_CALLER = r"""
#include <stdio.h>
#include "spmd_b200.h"
int main(void) {
  int64_t n = 8, st = 1;
  const float *in[1] = {(const float *)0x1000};
  int32_t bad[] = {SPMDB200_MAP_LOAD, 0, SPMDB200_MAP_NEG | 1 << 8 | 1 << 16, 0, SPMDB200_MAP_STORE, 0};
  int a = spmdb200_forall_map(4, &n, 1, in, &st, (float *)0x2000, &st, bad, 3, NULL, 0, 2, NULL);
  int b = spmdb200_forall_map(1, &n, 1, in, &st, (float *)0x2000, &st, bad, 3, NULL, 0, 2, NULL);
  unsigned long long first = 1;
  int c = spmdb200_check_status(&first);
  printf("%d %d %d %llu %s\n", a, b, c, first, spmdb200_status_string(SPMDB200_ERR_BOUNDS));
  return 0;
}
"""


def test_c_program_links_and_calls_the_abi(tmp_path):
    """A C caller compiles against include/spmd_b200.h, links libspmdb200.so
    and gets the argument checks' statuses (no CUDA call is reached)."""
    import shutil
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = spmd_mod("_lib")
    src = tmp_path / "caller.c"
    src.write_text(C_CALLER)
    exe = tmp_path / "caller"
    pkg = lib.PKG_DIR
    r = subprocess.run([cc, "-std=c11", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(src), "-o", str(exe),
                        f"-L{pkg}", "-lspmdb200", f"-Wl,-rpath,{pkg}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    a, b, c, first, *msg = out.stdout.split()
    assert int(a) == -1        # rank 4: invalid argument
    assert int(b) == -1        # register 1 read before it is written
    assert int(c) == -4 and int(first) == 0  # a release build has no out-of-range record
    assert "checked build" in " ".join(msg)
