"""Build libsvla.so in-tree with nvcc for sm_100a.

    python -m smolvla_mujoco_libero_b200.build [--debug]

The library lands next to this file so that it travels with the source tree.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libsvla.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


BUILD = PKG / "_build"
HEADER = PKG.parent / "include" / "svla.h"
FLAGS = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC"]


def units() -> list[tuple[Path, list[Path]]]:
    """(source, the files its object depends on) for every translation unit of the library."""
    kernels = [CSRC / "svla.cu", *sorted(CSRC.glob("*.cuh")), HEADER]
    return [(CSRC / "svla.cu", kernels), (CSRC / "engine.cpp", [CSRC / "engine.cpp", HEADER])]


def sources() -> list[Path]:
    return sorted({p for _, deps in units() for p in deps})


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def up_to_date() -> bool:
    return not _stale(OUT, sources())


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    if not force and not debug and up_to_date():
        return OUT
    BUILD.mkdir(exist_ok=True)
    objs = []
    for src, deps in units():
        obj = BUILD / (src.stem + (".debug.o" if debug else ".o"))
        if force or debug or _stale(obj, deps):
            cmd = [nvcc(), *FLAGS, "-c", "-o", str(obj), str(src)]
            if debug:
                cmd.insert(1, "-DSVLA_BOUNDS_CHECK")
            if verbose:
                cmd.append("-Xptxas=-v")
            subprocess.run(cmd, check=True)
        objs.append(str(obj))
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(OUT), *objs], check=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, debug=a.debug, verbose=a.verbose))
    sys.exit(0)
