"""spmdb200_sum_f32_noalloc: the deterministic f32 sum for callers that cannot
allocate device memory (code inside a stream capture that must not allocate,
a plugin whose host application owns every device allocation).  It keeps its
scratch in a fixed __device__ array inside the library instead of a caller
workspace.  Called through the C ABI and compared with spmdb200_sum_f32 (the
entry that takes a caller-provided workspace) on two calls in a row.

The file name sorts last so a run that stops at the first failure has already
run every other test; it also passes on its own in a fresh process."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import spmd_mod

pytestmark = pytest.mark.gpu

REL = 1e-6  # the f32-sum tolerance every reduction test uses


def _call_pair(lib, t, ws, n, off=0, stride=1):
    """spmdb200_sum_f32 (caller workspace) and spmdb200_sum_f32_noalloc on the
    view t[off : off + n*stride : stride], each into a zeroed output."""
    import torch
    c_i, c_p = ctypes.c_int64, ctypes.c_void_p
    a = (c_p(t.data_ptr()), c_p(t.data_ptr()), c_i(off), c_i(n), c_i(stride))
    ref = torch.zeros(1, device="cuda")
    got = torch.zeros(1, device="cuda")
    s = c_p(torch.cuda.current_stream().cuda_stream)
    st = lib.spmdb200_sum_f32(*a, c_p(ref.data_ptr()), c_p(ref.data_ptr()), c_i(0), c_i(n),
                              c_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), s)
    assert st == 0, lib.spmdb200_last_error_message()
    st = lib.spmdb200_sum_f32_noalloc(*a, c_p(got.data_ptr()), c_p(got.data_ptr()), c_i(0), c_i(n), s)
    assert st == 0, lib.spmdb200_last_error_message()
    torch.cuda.synchronize()
    return float(ref.item()), float(got.item())


# (n, offset, stride): unit-stride aligned views take the shared-memory-staged
# kernel; an odd offset (4-byte aligned only) or a stride of 2 takes the
# grid-stride kernel with the last-block ticket; n = 0 launches with no input.
CASES = [(1, 0, 1), (1000, 0, 1), (65537, 0, 1), (1 << 24, 0, 1),
         (65537, 1, 1), (1 << 20, 1, 1), (65537, 0, 2), (1 << 20, 3, 2), (0, 0, 1)]


@pytest.mark.parametrize("n,off,stride", CASES)
def test_noalloc_sum_matches_workspace_entry_twice(n, off, stride):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = spmd_mod("_lib").lib()
    total = off + max(n, 1) * stride
    a = np.random.RandomState(0).random_sample(total).astype(np.float32)
    t = torch.from_numpy(a).cuda()
    view = a[off:off + n * stride:stride] if n else a[:0]
    ws = torch.zeros(int(lib.spmdb200_sum_workspace_bytes(ctypes.c_int64(n))), dtype=torch.uint8, device="cuda")
    f64 = float(np.sum(view.astype(np.float64)))
    for _ in range(2):  # two calls in a row: the shared scratch must not carry state over
        ref, got = _call_pair(lib, t, ws, n, off, stride)
        assert abs(got - ref) <= REL * abs(ref)
        assert abs(got - f64) <= REL * abs(f64)
        if n == 0:
            assert got == 0.0 and ref == 0.0


def test_noalloc_rejects_bad_arguments():
    lib = spmd_mod("_lib").lib()
    c_i, c_p = ctypes.c_int64, ctypes.c_void_p
    fake = c_p(0x1000)
    st = lib.spmdb200_sum_f32_noalloc(fake, fake, c_i(0), c_i(10), c_i(1), fake, fake, c_i(0), c_i(-1), None)
    assert st == -1 and lib.spmdb200_last_error_message()
    st = lib.spmdb200_sum_f32_noalloc(fake, fake, c_i(0), c_i(10), c_i(1), None, None, c_i(0), c_i(10), None)
    assert st == -1
