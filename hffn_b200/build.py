"""In-tree build of ``hffn_b200/lib/libhffn_b200.so`` with nvcc for sm_100a (no JIT cache, no torch extension).

``build()`` compiles every ``csrc/*.cu`` into one shared library exporting the C ABI of ``include/hffn_b200.h``;
it rebuilds only when a source or header is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
LIB = HERE / "lib" / "libhffn_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    inputs = sources() + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > built for p in inputs)


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise FileNotFoundError("nvcc not found")
    return found


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB.parent.mkdir(exist_ok=True)
    partial = LIB.with_suffix(f".{os.getpid()}.tmp")
    command = [nvcc(), *ARCH, *FLAGS, "-o", str(partial), *map(str, sources())]
    if verbose:
        command.insert(1, "-Xptxas=-v")
    subprocess.run(command, check=True)
    partial.rename(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
