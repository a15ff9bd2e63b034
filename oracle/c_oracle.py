"""ctypes wrapper of the C oracle (``oracle/rvq_oracle.c``): TEST INFRASTRUCTURE ONLY.

Used by the tests as a fast full-size checker and by ``bench.py`` as the timed
CPU baseline (the reference's dequantise-then-matmul algorithm on host cores).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "librvq_oracle.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = ctypes.CDLL(str(LIB))
        vp = ctypes.c_void_p
        i64 = ctypes.c_int64
        lib.rvq_oracle_forward_group.argtypes = [ctypes.POINTER(vp), ctypes.c_int, vp, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, vp, i64, i64, vp, i64, vp, vp, i64, i64, ctypes.c_int]
        lib.rvq_oracle_reconstruct_group.argtypes = [ctypes.POINTER(vp), ctypes.c_int, vp, ctypes.c_int,
                                                     ctypes.c_int, ctypes.c_int, vp, i64, i64, vp, ctypes.c_int]
        lib.rvq_oracle_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(load().rvq_oracle_max_threads())


def _group_args(g: dict):
    if g.get("stage_scales") is not None:
        raise ValueError("the C restatement covers unscaled stages only; use rvq_oracle for stage scales")
    ids = [np.ascontiguousarray(a) for a in g["stage_ids"]]
    idw = 1 if ids[0].dtype == np.uint8 else 2
    ids = [a if idw == 1 else a.view(np.uint16) for a in ids]
    books = np.ascontiguousarray(np.stack([np.asarray(b, dtype=np.float16) for b in g["codebooks"]])).view(np.uint16)
    rho = np.ascontiguousarray(np.asarray(g["row_scale"], dtype=np.float16).reshape(-1)).view(np.uint16)
    ptrs = (ctypes.c_void_p * len(ids))(*[a.ctypes.data for a in ids])
    return ids, idw, books, rho, ptrs


def forward(x_bits: np.ndarray, groups: list[dict], in_features: int, bias_bits: np.ndarray | None = None,
            threads: int = 0) -> np.ndarray:
    """fp32 result of the per_group forward for all groups (rows concatenated)."""
    lib = load()
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M = x.shape[0]
    N = sum(int(np.asarray(g["row_scale"]).reshape(-1).shape[0]) for g in groups)
    y = np.zeros((M, N), dtype=np.float32)
    b = None if bias_bits is None else np.ascontiguousarray(bias_bits, dtype=np.uint16)
    row0 = 0
    for g in groups:
        ids, idw, books, rho, ptrs = _group_args(g)
        rows = rho.shape[0]
        R, entries, d = books.shape
        st = lib.rvq_oracle_forward_group(ptrs, idw, books.ctypes.data, R, entries, d, rho.ctypes.data, rows,
                                          in_features, x.ctypes.data, M, None if b is None else b.ctypes.data,
                                          y.ctypes.data, N, row0, threads)
        if st != 0:
            raise MemoryError("oracle forward failed")
        row0 += rows
    return y


def reconstruct(groups: list[dict], in_features: int, threads: int = 0) -> np.ndarray:
    lib = load()
    parts = []
    for g in groups:
        ids, idw, books, rho, ptrs = _group_args(g)
        rows = rho.shape[0]
        R, entries, d = books.shape
        w = np.zeros((rows, in_features), dtype=np.uint16)
        lib.rvq_oracle_reconstruct_group(ptrs, idw, books.ctypes.data, R, entries, d, rho.ctypes.data, rows,
                                         in_features, w.ctypes.data, threads)
        parts.append(w)
    return np.concatenate(parts, axis=0)
