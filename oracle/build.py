"""Builds the CPU oracle oracle/_build/libspmd_oracle.so (test infrastructure).

    python oracle/build.py [--force]

gcc -O3 -fopenmp -ffp-contract=off: no fused multiply-add and no fast-math,
so every f32 operation rounds exactly as written in spmd_oracle.c.
-march=x86-64-v3 (AVX2) keeps the binary portable to any current x86 server
the GPU runs are hosted on.
"""
from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "spmd_oracle.c"
OUT = HERE / "_build" / "libspmd_oracle.so"
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
          "-fPIC", "-shared", "-std=c11", "-Wall", "-Wno-unused-parameter"]


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if force or not OUT.exists() or OUT.stat().st_mtime < SRC.stat().st_mtime:
        cc = shutil.which("gcc") or "cc"
        r = subprocess.run([cc, *CFLAGS, "-o", str(OUT), str(SRC), "-lm"], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    print(build(force=ap.parse_args().force))
    sys.exit(0)
