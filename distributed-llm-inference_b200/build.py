"""Build libpaged_decode_b200.so in-tree with nvcc for sm_100a.

The library has no PyTorch dependency: it is plain CUDA C++ behind the
`extern "C"` API of include/paged_decode_b200.h, with the CUDA runtime
linked statically so that it loads next to any PyTorch build.

Usage: python -m <package>.build   (or call build_library()).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_NAME = "libpaged_decode_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-shared",
    "-cudart", "static",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the paged-decode library needs the CUDA toolkit to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [
        REPO_ROOT / "include" / "paged_decode_b200.h"]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in sources())


def build_library(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile csrc/paged_decode.cu (which includes every kernel) into LIB_PATH."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, *(extra_flags or []), "-I", str(REPO_ROOT / "include"),
           str(CSRC / "paged_decode.cu"), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout, proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose=True,
                  extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB_PATH)
