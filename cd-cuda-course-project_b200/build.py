"""
build.py — nvcc recipes for the in-tree sm_100a shared libraries.

The reference compiles one standalone executable per variant with
``nvcc -O3 -arch=sm_75 --use_fast_math -Xptxas -v`` (autotune.py:120-129,
src/benchmark.py:109-130). Here every build is a position-independent shared
library for ``sm_100a`` exporting the C ABI of ``include/kt_abi.h``; fast-math
is never used (the parity budgets are 1e-5 relative for fp32 softmax/LN).
``-Xptxas -v`` is kept: its resource lines feed ``occupancy.py``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import tempfile
from pathlib import Path
from typing import Iterable, Optional

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB_DIR = PKG / "lib"
DEFAULT_SRC = CSRC / "libkt.cu"
DEFAULT_LIB = LIB_DIR / "libkt.so"
DEFAULT_PTXAS_LOG = LIB_DIR / "libkt.ptxas.txt"

ARCH = "sm_100a"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
BASE_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xptxas", "-v",
    "--shared",
    "-Xcompiler", "-fPIC",
    # hidden by default: only the KT_API entry points are exported, so the
    # C++ internals of two loaded variants (including function-local statics,
    # which GCC would otherwise make process-unique) never bind to each other
    "-Xcompiler", "-fvisibility=hidden",
]


def nvcc_path() -> str:
    """Locate nvcc (PATH first, then the standard CUDA prefix)."""
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path("/usr/local/cuda/bin/nvcc")
    if cand.exists():
        return str(cand)
    raise FileNotFoundError("nvcc not found (PATH or /usr/local/cuda/bin)")


def nvcc_command(src: Path, out: Path, defines: Optional[dict] = None,
                 extra_flags: Optional[Iterable[str]] = None) -> list[str]:
    """Full nvcc command line for one shared library."""
    cmd = [nvcc_path(), *ARCH_FLAGS, *BASE_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}"]
    for key, val in (defines or {}).items():
        cmd.append(f"-D{key}" if val is None else f"-D{key}={val}")
    if extra_flags:
        cmd.extend(extra_flags)
    cmd += [str(src), "-o", str(out)]
    return cmd


def compile_shared(src: Path, out: Path, defines: Optional[dict] = None,
                   extra_flags: Optional[Iterable[str]] = None,
                   timeout: int = 900) -> tuple[bool, str]:
    """
    Compile ``src`` into the shared library ``out``.

    The library is written to a temporary name and renamed into place, so a
    concurrent loader never sees a half-written file. Returns (ok, stderr);
    stderr carries the ptxas resource report.
    """
    out = Path(out)
    out.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=out.stem + ".", suffix=".so.tmp", dir=str(out.parent))
    os.close(fd)
    try:
        cmd = nvcc_command(Path(src), Path(tmp), defines, extra_flags)
        proc = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
        if proc.returncode != 0:
            return False, proc.stderr + proc.stdout
        os.replace(tmp, out)
        return True, proc.stderr
    except subprocess.TimeoutExpired as exc:
        return False, f"nvcc timed out after {timeout}s: {exc}"
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def _sources() -> list[Path]:
    files = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return [f for f in files if f.is_file()]


def default_library_stale() -> bool:
    """True when libkt.so is missing or older than any source it is built from."""
    if not DEFAULT_LIB.exists():
        return True
    built = DEFAULT_LIB.stat().st_mtime
    return any(f.stat().st_mtime > built for f in _sources())


def build_default(force: bool = False) -> Path:
    """Build (if stale) and return the path of the default library."""
    if force or default_library_stale():
        ok, log = compile_shared(DEFAULT_SRC, DEFAULT_LIB)
        if not ok:
            raise RuntimeError(f"building {DEFAULT_LIB.name} failed:\n{log}")
        DEFAULT_PTXAS_LOG.write_text(log)
    return DEFAULT_LIB


if __name__ == "__main__":
    import sys
    path = build_default(force="--force" in sys.argv)
    print(path)
