"""spmd-dialect_b200: B200 (sm_100a) kernels for the three kernel families
spmd-dialect's SPMDToGPU lowering emits -- elementwise foralls, promoted
stencil sweeps (3-point, Jacobi-2D, Jacobi-3D) and hierarchical reductions --
behind the C ABI of include/spmd_b200.h.

Layout of the package:
    csrc/            CUDA kernels (sm_100a) and the C ABI (api.cu)
    build.py         nvcc build of libspmdb200.so + spmdb200_kernels.cubin
    _lib.py          ctypes binding of the C ABI (no fallback: raises if missing)
    kernels.py       device entries over torch tensors
    host.py          host-buffer entries in harness/run_host.py's convention
    cuda_driver.py   driver-API client with harness/cuda_driver.py's surface,
                     for loading spmdb200_kernels.cubin by kernel name
    slab.py          multi-GPU row-slab Jacobi-2D (one process per GPU)

Import with importlib (the directory name has a hyphen):
    spmd = importlib.import_module("spmd-dialect_b200")
"""
from ._lib import CUBIN_PATH, LIB_PATH, SpmdError, lib

__all__ = ["CUBIN_PATH", "LIB_PATH", "SpmdError", "lib", "version"]


def version() -> str:
    return lib().spmdb200_version().decode()
