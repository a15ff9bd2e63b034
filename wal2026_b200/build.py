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


# translation units: (source, extra defines).  The GEMV source is compiled once
# per block size and weight type so the template instantiations build in
# parallel, plus once for its C entry points.
def units() -> list[tuple[Path, list[str]]]:
    out = []
    for src in sources():
        if src.name == "wal_rvq_gemv.cu":
            out.append((src, ["-DWAL_UNIT_API"]))
            out += [(src, [f"-DWAL_UNIT_D={d}", f"-DWAL_UNIT_T={t}"]) for t in (0, 1) for d in (8, 16, 32)]
        else:
            out.append((src, []))
    return out


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return res.stdout + res.stderr


def build(verbose: bool = False, extra: list[str] | None = None, force: bool = False) -> Path:
    from concurrent.futures import ThreadPoolExecutor

    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    common = [_nvcc(), *(extra or []), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}"]
    jobs = []
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    for src, defs in units():
        tag = "_".join(d.split("=")[-1] if "=" in d else d[2:].lower() for d in defs)
        obj = objdir / (f"{src.stem}_{tag}.o" if tag else f"{src.stem}.o")
        cmd = common + defs + ["-c", str(src), "-o", str(obj)]
        stamp = obj.with_suffix(".cmd")
        # an object is reused when it is newer than its source and every header
        # and was built by the same command line
        fresh = (not force and obj.exists() and stamp.exists() and stamp.read_text() == " ".join(cmd)
                 and all(p.stat().st_mtime <= obj.stat().st_mtime for p in [src, *headers]))
        jobs.append((cmd, obj, stamp, fresh))
    todo = [j for j in jobs if not j[3]]

    def compile_one(job):
        out = _run(job[0], verbose)
        job[2].write_text(" ".join(job[0]))
        return out

    with ThreadPoolExecutor(max_workers=max(1, min(len(todo) or 1, os.cpu_count() or 1))) as ex:
        logs = list(ex.map(compile_one, todo))
    if verbose:
        print("".join(logs), file=sys.stderr)
    link = [_nvcc(), *ARCH, "-shared", "-o", str(LIB) + ".tmp", *[str(j[1]) for j in jobs], "-lcuda"]
    _run(link, verbose)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


def ensure_built() -> Path:
    if _stale():
        build()
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv))
