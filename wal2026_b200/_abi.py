"""ctypes binding of the C ABI in ``include/wal_rvq.h`` (library ``libwal_rvq.so``).

The library is loaded from this package directory.  There is no fallback: if
it is missing or does not load, every compute entry point raises, so a machine
without the CUDA build can never silently run a CPU path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libwal_rvq.so"

WAL_OK = 0
WAL_ERR_INVALID_ARGUMENT = 1
WAL_ERR_SHAPE = 2
WAL_ERR_ALIGNMENT = 3
WAL_ERR_ID_RANGE = 4
WAL_ERR_UNSUPPORTED = 5
WAL_ERR_CUDA = 6
WAL_ERR_BUFFER_TOO_SMALL = 7
WAL_ERR_PEER_TIMEOUT = 8

WAL_MAX_RANKS = 8
WAL_IPC_HANDLE_BYTES = 64

WAL_BF16 = 0
WAL_F32 = 1
WAL_F16 = 2

WAL_SUM_EXACT = 0
WAL_SUM_FAST = 1

DTYPE_CODE = {torch.bfloat16: WAL_BF16, torch.float32: WAL_F32, torch.float16: WAL_F16}

# every function the header declares, with its ctypes signature
_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_vp = ctypes.c_void_p


class Geometry(ctypes.Structure):
    _fields_ = [
        ("out_features", ctypes.c_int64),
        ("in_features", ctypes.c_int64),
        ("block_size", ctypes.c_int32),
        ("num_stages", ctypes.c_int32),
        ("num_entries", ctypes.c_int32),
        ("num_groups", ctypes.c_int32),
    ]


class Layer(ctypes.Structure):
    _fields_ = [
        ("geom", Geometry),
        ("num_tiles", ctypes.c_int64),
        ("packed_ids", ctypes.c_void_p),
        ("tile_table", ctypes.c_void_p),
        ("codebooks", ctypes.c_void_p),
        ("row_scale", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("group_rows", ctypes.POINTER(ctypes.c_int64)),
        ("stage_scales", ctypes.c_void_p),
        ("sum_mode", ctypes.c_int32),
    ]


class Corrections(ctypes.Structure):
    """``wal_rvq_corrections``: device buffers of the per-block corrections of one linear."""
    _fields_ = [
        ("group_flags", ctypes.c_void_p),
        ("residual_signs", ctypes.c_void_p),
        ("residual_scale", ctypes.c_void_p),
        ("block_scale", ctypes.c_void_p),
        ("sign_matrix", ctypes.c_void_p),
        ("transform", ctypes.c_void_p),
        ("transform_bias", ctypes.c_void_p),
    ]


WAL_CORR_SIGN = 1
WAL_CORR_BLOCK_SCALE = 2
WAL_CORR_MATRIX = 4
WAL_CORR_POLAR = 8
WAL_CORR_BIAS = 16


class TPPush(ctypes.Structure):
    """``wal_tp_push``: where a row-parallel GEMV stores its tagged partial."""
    _fields_ = [
        ("num_ranks", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("dst", ctypes.c_void_p * WAL_MAX_RANKS),
        ("ld_dst", ctypes.c_int64),
        ("epoch", ctypes.c_void_p),
    ]


class IDRouteLayer(ctypes.Structure):
    """``wal_idroute_layer``: device buffers of one ID-route linear."""
    _fields_ = [
        ("out_features", ctypes.c_int64),
        ("in_features", ctypes.c_int64),
        ("num_routes", ctypes.c_int32),
        ("packed_ids", ctypes.c_void_p),
        ("codebook_sum", ctypes.c_void_p),
        ("row_scale", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
    ]


_GP = ctypes.POINTER(Geometry)
_LP = ctypes.POINTER(Layer)

SIGNATURES: dict[str, tuple] = {
    "wal_status_string": (ctypes.c_char_p, [_c_int]),
    "wal_version": (_c_int, []),
    "wal_rvq_packed_size": (_c_int, [_GP, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_size_t),
                                     ctypes.POINTER(ctypes.c_int64)]),
    "wal_rvq_pack": (_c_int, [_GP, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(_vp), _vp, ctypes.c_size_t,
                              ctypes.POINTER(ctypes.c_int32)]),
    "wal_route_pack": (_c_int, [_GP, _vp, _vp, _vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32)]),
    "wal_rvq_gemv": (_c_int, [_LP, _vp, _c_i64, _c_i64, _vp, _c_i64, _c_int, _vp]),
    "wal_rvq_gemv_typed": (_c_int, [_LP, _vp, _c_int, _c_i64, _c_i64, _vp, _c_i64, _c_int, _c_int, _c_int, _vp]),
    "wal_rvq_dequant_typed": (_c_int, [_LP, _vp, _c_i64, _c_int, _vp]),
    "wal_rvq_assign": (_c_int, [_vp, _c_i64, ctypes.c_int32, _vp, ctypes.c_int32, _vp, _vp, _vp]),
    "wal_rvq_gemv_corrected": (_c_int, [_LP, ctypes.POINTER(Corrections), _vp, _c_int, _c_i64, _c_i64, _vp, _c_i64,
                                        _c_int, _vp]),
    "wal_rvq_dequant_corrected": (_c_int, [_LP, ctypes.POINTER(Corrections), _vp, _c_i64, _c_int, _vp]),
    "wal_rvq_gemm_typed": (_c_int, [_LP, _vp, _c_int, _c_i64, _c_i64, _vp, _c_i64, _c_int, _vp, _vp]),
    "wal_rvq_gemv_ex": (_c_int, [_LP, _vp, _c_i64, _c_i64, _vp, _c_i64, _c_int, _c_int, _c_int, _vp]),
    "wal_rvq_gemm": (_c_int, [_LP, _vp, _c_i64, _c_i64, _vp, _c_i64, _c_int, _vp, _vp]),
    "wal_rvq_dequant": (_c_int, [_LP, _vp, _c_i64, _vp]),
    "wal_rvq_unpack_ids": (_c_int, [_LP, _vp, _vp]),
    "wal_idroute_packed_size": (_c_int, [_c_i64, _c_i64, ctypes.POINTER(ctypes.c_size_t)]),
    "wal_idroute_pack": (_c_int, [_c_i64, _c_i64, ctypes.c_int32, _vp, _vp, ctypes.c_size_t]),
    "wal_idroute_gemv": (_c_int, [ctypes.POINTER(IDRouteLayer), _vp, _c_i64, _c_i64, _vp, _c_i64, _c_int, _vp]),
    "wal_idroute_dequant": (_c_int, [ctypes.POINTER(IDRouteLayer), _vp, _c_i64, _c_int, _vp]),
    "wal_decode_attention_workspace": (ctypes.c_size_t, [_c_i64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                         _c_i64]),
    "wal_decode_attention": (_c_int, [_vp, _c_i64, _vp, _vp, _c_i64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                      _c_i64, _c_i64, ctypes.c_float, _vp, _c_i64, _vp, ctypes.c_size_t, _vp]),
    "wal_decode_attention_ex": (_c_int, [_vp, _c_i64, _vp, _vp, _c_i64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                         _c_i64, _c_i64, ctypes.c_float, _vp, _c_i64, _vp, ctypes.c_size_t, _c_int,
                                         _vp]),
    "wal_decode_attention_static": (_c_int, [_vp, _c_i64, _vp, _vp, _c_i64, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.c_int32, _c_i64, _c_i64, ctypes.c_float, _vp, _c_i64, _vp]),
    "wal_tp_push_rows": (_c_int, [_vp, _c_i64, _c_int, _c_i64, _c_i64, ctypes.POINTER(TPPush), _vp]),
    "wal_rvq_gemv_push": (_c_int, [_LP, _vp, _c_i64, _c_i64, ctypes.POINTER(TPPush), _vp]),
    "wal_tp_reduce_rmsnorm": (_c_int, [_vp, ctypes.c_int32, _c_i64, _c_i64, _vp, _vp, _vp, _c_i64, _vp,
                                       ctypes.c_float, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp]),
    "wal_residual_rmsnorm": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, ctypes.c_float, _vp, _c_i64, _c_i64, _c_i64,
                                      _vp]),
    "wal_rope_kv_append": (_c_int, [_vp, _c_i64, _c_i64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _vp, _vp,
                                    _c_i64, _vp, _vp, _vp, _c_i64, _vp]),
    "wal_silu_mul": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _vp, _c_i64, _vp]),
    "wal_peer_region_create": (_c_int, [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]),
    "wal_peer_region_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "wal_peer_region_close": (_c_int, [_vp]),
    "wal_peer_region_free": (_c_int, [_vp]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises RuntimeError when it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built; run `python -m wal2026_b200.build` (nvcc, sm_100a). "
            "This package has no CPU fallback."
        )
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


class WalError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        text = load().wal_status_string(status).decode()
        super().__init__(f"{where}: {text} (status {status})")


class WalValueError(ValueError):
    def __init__(self, status: int, where: str):
        self.status = status
        text = load().wal_status_string(status).decode()
        super().__init__(f"{where}: {text} (status {status})")


def check(status: int, where: str) -> None:
    """Map a wal_status to the exception the reference raises for the same condition."""
    if status == WAL_OK:
        return
    if status in (WAL_ERR_CUDA, WAL_ERR_PEER_TIMEOUT):
        raise WalError(status, where)
    raise WalValueError(status, where)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device | None = None) -> int:
    """The cudaStream_t of torch's current stream on ``device`` (default: the current device)."""
    if _raw_stream is not None:  # a fraction of a microsecond instead of ~3 us through the Stream object
        idx = torch.cuda.current_device() if device is None or device.index is None else device.index
        return int(_raw_stream(idx))
    return int(torch.cuda.current_stream(device).cuda_stream)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else int(t.data_ptr())
