"""Build the in-tree CUDA/C++ library ``libwal_rvq.so`` for sm_100a with nvcc.

The library is built next to this file so that it travels with the source tree
(no site-packages install, no JIT cache).  ``python -m wal2026_b200.build``
rebuilds it; ``ensure_built()`` rebuilds only when a source is newer than the
library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libwal_rvq.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libwal_rvq.so")
    return cand


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    cmd = [
        _nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}", "-o", str(LIB) + ".tmp",
        *[str(s) for s in sources()], "-lcuda",
    ]
    if extra:
        cmd[1:1] = extra
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


def ensure_built() -> Path:
    if _stale():
        build()
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
