"""Build the in-tree CUDA library ``libdels_b200.so`` (sm_100a only).

The library is compiled with nvcc directly from ``csrc/`` into this package directory,
so it travels with the source tree and is found by :mod:`dels_b200._lib` without any
install step.  ``python -m dels_b200.build`` (with ``dels-spec_b200`` on ``sys.path``)
or ``__graft_entry__.build()`` runs it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
REPO_ROOT = PKG_DIR.parent.parent
INCLUDE_DIR = REPO_ROOT / "include"
LIB_NAME = "libdels_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ["api.cu", "small_kernels.cu", "f32_score.cu", "runner_kernels.cu"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-shared",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin directory on PATH")
    return cand


def _inputs() -> list[Path]:
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh"))
    files.append(INCLUDE_DIR / "dels_b200.h")
    files.append(Path(__file__).resolve())
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > built for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``libdels_b200.so`` if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *GENCODE, *NVCC_FLAGS, "-I", str(INCLUDE_DIR)]
    cmd += [str(CSRC / s) for s in SOURCES]
    cmd += ["-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
