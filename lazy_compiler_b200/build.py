"""Builds ``liblazyb200.so`` in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` file is compiled to an object in ``_build/`` (in
parallel, skipped when the object is newer than its sources) and linked into
``lazy_compiler_b200/liblazyb200.so`` with the CUDA runtime linked
statically, so the library only needs the driver at run time.
``python -m lazy_compiler_b200.build`` runs it from the command line.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "liblazyb200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build liblazyb200.so")
    return path


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [d.stat().st_mtime for d in _deps()])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{result.stderr}")
    if verbose and result.stderr:
        print(result.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every kernel source and link the shared library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if force:
        for obj in BUILD.glob("*.o"):
            obj.unlink()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), sources))
    newest = max(o.stat().st_mtime for o in objects)
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest or force:
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-cudart", "static"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"link failed:\n{result.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv))
