"""Build the in-tree native library ``_lib/libnvfp4_qsa.so`` with nvcc for sm_100a.

Usage: ``python -m nvfp4_qsa._build [--force]`` (with ``nvfp4-qsa_b200`` on
``sys.path``), or ``__graft_entry__.build()``.  The library carries every CUDA
kernel of this package behind the C ABI declared in ``include/nvfp4_qsa.h``.
It is compiled without fast-math: the writer's bytes must match the reference
codec bit for bit, which needs IEEE division and no multiply-add contraction.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
SOURCE_DIR = PACKAGE_DIR.parent / "csrc"
INCLUDE_DIR = PACKAGE_DIR.parent.parent / "include"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_NAME = "libnvfp4_qsa.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-shared"]


def library_path() -> Path:
    return LIB_DIR / LIB_NAME


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the NVFP4 QSA CUDA library cannot be built")


def _sources() -> list[Path]:
    return sorted(SOURCE_DIR.glob("*.cu"))


def _inputs() -> list[Path]:
    return _sources() + sorted(SOURCE_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def is_stale() -> bool:
    lib = library_path()
    if not lib.exists():
        return True
    built = lib.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile all ``csrc/*.cu`` into one shared library; returns its path."""
    lib = library_path()
    if not force and not is_stale():
        return lib
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = lib.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE_DIR}", f"-I{SOURCE_DIR}",
           *map(str, _sources()), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
