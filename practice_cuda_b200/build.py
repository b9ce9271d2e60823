"""Build libpcb200.so in-tree with nvcc for sm_100a.

``python -m practice_cuda_b200.build [--force]``.  The library is rebuilt
when any source under ``csrc/`` or ``include/`` is newer than it.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "pcb200.cu")
OUT = os.path.join(HERE, "_lib", "libpcb200.so")
PROF_OUT = os.path.join(HERE, "_lib", "libpcb200_prof.so")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-shared",
]


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def needs_build(path: str = OUT) -> bool:
    if not os.path.exists(path):
        return True
    t = os.path.getmtime(path)
    return any(os.path.getmtime(s) > t for s in _sources())


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libpcb200")
    return path


def build(force: bool = False, verbose: bool = False, profiling: bool = False, out: str | None = None) -> str:
    """Build the library.  ``profiling`` compiles the PCB200_PROFILING
    switches in (environment knobs that change kernel selection or skip work;
    never shipped) into ``out`` (default ``_lib/libpcb200_prof.so``)."""
    dst = out or (PROF_OUT if profiling else OUT)
    if not force and not needs_build(dst):
        return dst
    os.makedirs(os.path.dirname(dst), exist_ok=True)
    tmp = dst + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, *(["-DPCB200_PROFILING"] if profiling else []), "-o", tmp, SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, dst)
    return dst


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--profiling", action="store_true", help="build libpcb200_prof.so with -DPCB200_PROFILING")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, profiling=args.profiling))
