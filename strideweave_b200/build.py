"""Build recipe of the native library ``strideweave_b200/_lib/libswb200.so``.

Compiles every CUDA translation unit under ``csrc/`` for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into one shared object that
exports the C ABI declared in ``include/strideweave_b200.h``.  Run
``python -m strideweave_b200.build`` (or ``__graft_entry__.build()``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_PATH = LIB_DIR / "libswb200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    """Return the nvcc executable (CUDA_HOME first, then PATH)."""
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: the B200 carrier library cannot be built")
    return found


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def needs_rebuild() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    inputs = list(sources()) + list(CSRC_DIR.glob("*.cuh")) + list(INCLUDE_DIR.glob("*.h"))
    return any(p.stat().st_mtime > built for p in inputs)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not needs_rebuild():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "-rdc=true",
        "-shared",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-Xptxas",
        "-v" if verbose else "-O3",
        f"-I{INCLUDE_DIR}",
        f"-I{CSRC_DIR}",
        *[str(s) for s in sources()],
        "-o",
        str(tmp),
    ]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(
            "nvcc failed building the B200 carrier library:\n"
            + result.stdout
            + result.stderr
        )
    if verbose:
        sys.stderr.write(result.stdout + result.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv))
