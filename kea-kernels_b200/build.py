"""Builds libkea_lowbit.so (sm_100a) into the kea_kernels package directory with nvcc.

Usage: python kea-kernels_b200/build.py [--force]
The library is compiled in-tree so it travels with the source tree; nothing is JIT-compiled at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OUT = HERE / "kea_kernels" / "libkea_lowbit.so"
SOURCES = [CSRC / "kea_lowbit.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "kea_lowbit.h"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or add the CUDA toolkit to PATH")


def command() -> list[str]:
    return [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
            "-fmad=false", "-Xptxas", "-v", f"-I{ROOT / 'include'}", "-Xcompiler", "-fPIC,-O2", "-shared",
            "-o", str(OUT), *map(str, SOURCES)]


def stale() -> bool:
    if not OUT.exists():
        return True
    built = OUT.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    if force or stale():
        cmd = command()
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
        if verbose:
            print(res.stderr)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
