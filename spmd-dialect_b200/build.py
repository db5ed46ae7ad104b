"""Builds libspmdb200.so and spmdb200_kernels.cubin in place (sm_100a only).

    python spmd-dialect_b200/build.py [--force] [-j N] [--no-checked]

Each csrc/*.cu except refabi.cu is compiled to an object under _build/ and
linked with the static CUDA runtime into libspmdb200.so (no link-time
dependency on libcuda, so the library also loads on machines without a GPU
driver).  refabi.cu -- the kernels with the reference's PTX entry names -- is
compiled to spmdb200_kernels.cubin for cuModuleLoadData callers.
libspmdb200_checked.so is the same library with the general kernels
(forall_map.cu, stencil_nd.cu) compiled with -DSPMDB200_CHECKED.  ptxas
register / spill reports go to _build/ptxas.log.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libspmdb200.so"
# The checked variant: the general kernels rebuilt with run-time index checks
# that record instead of trapping (and NaN-poisoned shared tiles), linked with
# the release objects of every other file.  Loaded when SPMDB200_VARIANT=checked.
CHECKED_LIB = PKG / "libspmdb200_checked.so"
CHECKED_UNITS = ("forall_map.cu", "stencil_nd.cu")
CUBIN = PKG / "spmdb200_kernels.cubin"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2", "-Xptxas", "-v", f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the B200 kernels cannot be built")


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> str:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, checked: bool = True) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    deps = _deps()
    units = [p for p in sorted(CSRC.glob("*.cu")) if p.name != "refabi.cu"]
    objs = [BUILD / (p.stem + ".o") for p in units]
    todo = [(u, o) for u, o in zip(units, objs) if force or _stale(o, [u] + deps)]
    logs: dict[str, str] = {}
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        futs = {ex.submit(_run, [cc, *NVCC_FLAGS, "-c", str(u), "-o", str(o)]): u for u, o in todo}
        cubin_src = CSRC / "refabi.cu"
        if force or _stale(CUBIN, [cubin_src] + deps):
            futs[ex.submit(_run, [cc, *NVCC_FLAGS, "-cubin", str(cubin_src), "-o", str(CUBIN)])] = cubin_src
        for f in cf.as_completed(futs):
            logs[futs[f].name] = f.result()
    if force or todo or _stale(LIB, objs):
        _run([cc, "-shared", *ARCH, "-cudart", "static", "-Xcompiler", "-fPIC", "-o", str(LIB),
              *map(str, objs), "-lpthread", "-ldl", "-lrt"])
    if checked:
        cdir = BUILD / "checked"
        cdir.mkdir(exist_ok=True)
        cobjs = []
        with cf.ThreadPoolExecutor(max_workers=len(CHECKED_UNITS)) as ex:
            futs = {}
            for name in CHECKED_UNITS:
                u, o = CSRC / name, cdir / (Path(name).stem + ".o")
                cobjs.append(o)
                if force or _stale(o, [u] + deps):
                    futs[ex.submit(_run, [cc, *NVCC_FLAGS, "-DSPMDB200_CHECKED", "-c", str(u), "-o", str(o)])] = u
            for f in cf.as_completed(futs):
                logs["checked/" + futs[f].name] = f.result()
        rest = [o for u, o in zip(units, objs) if u.name not in CHECKED_UNITS]
        if force or _stale(CHECKED_LIB, cobjs + rest):
            _run([cc, "-shared", *ARCH, "-cudart", "static", "-Xcompiler", "-fPIC", "-o", str(CHECKED_LIB),
                  *map(str, rest + cobjs), "-lpthread", "-ldl", "-lrt"])
    if logs:
        with open(BUILD / "ptxas.log", "a") as fh:
            for name, text in sorted(logs.items()):
                fh.write(f"==== {name}\n{text}\n")
    if verbose:
        for name, text in sorted(logs.items()):
            print(f"==== {name}\n{text}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--no-checked", action="store_true", help="skip libspmdb200_checked.so")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v, checked=not a.no_checked))


if __name__ == "__main__":
    sys.exit(main())
