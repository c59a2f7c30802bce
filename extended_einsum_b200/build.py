"""Builds the sm_100a shared library libxe_b200.so in-tree with nvcc.

The library is the C ABI declared in include/xe_b200.h; the Python package
loads it with ctypes (extended_einsum_b200/_lib.py).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
LIBRARY = PACKAGE_DIR / "libxe_b200.so"
SOURCES = [CSRC / "xe_b200.cu"]
DEPENDENCIES = sorted(CSRC.glob("*.cuh")) + [REPO_ROOT / "include" / "xe_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def find_nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def is_stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + DEPENDENCIES)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compiles libxe_b200.so for sm_100a if a source is newer than the library."""
    if not force and not is_stale():
        return LIBRARY
    cmd = [find_nvcc(), *NVCC_FLAGS, *(extra_flags or []), "-o", str(LIBRARY), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd[cmd.index(str(LIBRARY))] = str(tmp)
    subprocess.run(cmd, check=True, cwd=str(REPO_ROOT))
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, extra_flags=[a for a in sys.argv[1:] if a != "--force"])
