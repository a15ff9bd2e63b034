"""Host-side re-layout of Block-RVQ encodings into the packed, tile-major form.

The packed form (layout documented in ``include/wal_rvq.h``) is built once at
load time by the C ABI's ``wal_rvq_pack``/``wal_route_pack`` and then lives in
device memory as module buffers.  It replaces the per-stage id buffers of the
reference's ``PackedBlockRVQGroup`` (reference ``src/runtime.py:249-344``).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _abi
from .block_vq import BlockRVQEncoding, GroupedBlockRVQEncoding


@dataclass
class PackedArrays:
    """Host (CPU) tensors of one packed linear, ready to be registered as buffers."""

    geometry: _abi.Geometry
    num_tiles: int
    packed_ids: torch.Tensor  # uint8 [bytes]
    tile_table: torch.Tensor  # int32 [num_tiles, 4]
    codebooks: torch.Tensor   # fp16 [groups, R, entries, d]
    row_scale: torch.Tensor   # fp16 [N]
    stage_scales: Optional[torch.Tensor] = None  # fp32 [groups, R] per-stage scales


def _geometry(N: int, K: int, d: int, R: int, entries: int, groups: int) -> _abi.Geometry:
    return _abi.Geometry(out_features=N, in_features=K, block_size=d, num_stages=R, num_entries=entries,
                         num_groups=groups)


def validate_grouped(enc: GroupedBlockRVQEncoding, allow_corrections: bool = False) -> tuple[int, int, int, int]:
    """Check an encoding is supported by the packed path; return (d, R, entries, K).

    Unsupported encodings raise ``ValueError`` like the reference's fused path
    does (``src/runtime.py:848-853``).  Per-block corrections are accepted when
    ``allow_corrections`` (their side arrays come from ``pack_corrections``).
    """
    if not enc.groups:
        raise ValueError("encoding has no groups")
    K = int(enc.original_shape[1])
    first = enc.groups[0]
    d = int(first.block_size)
    R = int(first.num_stages)
    entries = int(first.codebooks[0].shape[0])
    row = 0
    for g, (r0, r1) in zip(enc.groups, enc.row_slices):
        if not g.is_plain() and not allow_corrections:
            raise ValueError("the packed id stream covers the stage sum only; pack the per-block corrections "
                             "(block_scale, residual correction, transform) with pack_corrections")
        if int(g.block_size) != d or int(g.num_stages) != R:
            raise ValueError("all row groups must share block_size and num_stages")
        if any(int(c.shape[0]) != entries or int(c.shape[1]) != d for c in g.codebooks):
            raise ValueError("all codebooks must be [entries, block_size] with the same entries")
        if int(g.original_shape[1]) != K:
            raise ValueError("group in_features differs from the layer's")
        if r0 != row or r1 - r0 != int(g.original_shape[0]):
            raise ValueError("row_slices must be contiguous and match the group row counts")
        if int(g.padded_cols) != -(-K // d) * d:
            raise ValueError("padded_cols must equal ceil(in_features / block_size) * block_size")
        row = r1
    if row != int(enc.original_shape[0]):
        raise ValueError("row_slices do not cover out_features")
    if d not in (8, 16, 32):
        raise ValueError(f"block_size {d} is not supported (8, 16 or 32)")
    if not 1 <= R <= 4:
        raise ValueError(f"num_stages {R} is not supported (1..4)")
    if R > 1 and entries > 256:
        raise ValueError("multi-stage codebooks must have <= 256 entries")
    if entries > 32767:
        raise ValueError("codebooks larger than 32767 entries are not supported")
    if K % 4 != 0:
        raise ValueError("in_features must be a multiple of 4")
    return d, R, entries, K


def _ids_array(t: torch.Tensor, entries: int) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if entries <= 256:
        if t.dtype != torch.uint8:
            t = t.to(torch.int64)
            if int(t.min()) < 0 or int(t.max()) >= 256:
                raise ValueError("id out of range of its codebook")
            t = t.to(torch.uint8)
        return t.numpy()
    # two-byte ids (int16 in the reference for <= 32767 entries)
    if t.dtype == torch.int16:
        return t.numpy().view(np.uint16)
    t = t.to(torch.int64)
    if int(t.min()) < 0 or int(t.max()) >= 65536:
        raise ValueError("id out of range of its codebook")
    return t.to(torch.int32).numpy().astype(np.uint16)


def pack_grouped(enc: GroupedBlockRVQEncoding, allow_corrections: bool = False) -> PackedArrays:
    d, R, entries, K = validate_grouped(enc, allow_corrections)
    lib = _abi.load()
    N = int(enc.original_shape[0])
    G = len(enc.groups)
    geom = _geometry(N, K, d, R, entries, G)
    rows = (ctypes.c_int64 * G)(*[int(g.original_shape[0]) for g in enc.groups])
    nbytes = ctypes.c_size_t(0)
    ntiles = ctypes.c_int64(0)
    _abi.check(lib.wal_rvq_packed_size(ctypes.byref(geom), rows, ctypes.byref(nbytes), ctypes.byref(ntiles)),
               "wal_rvq_packed_size")
    arrays = []
    for g in enc.groups:
        for ids in g.stage_ids:
            a = _ids_array(ids, entries)
            if a.shape != (int(g.original_shape[0]), -(-K // d)):
                raise ValueError(f"stage ids shape {a.shape} does not match [rows, blocks]")
            arrays.append(np.ascontiguousarray(a))
    ptrs = (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])
    packed = torch.empty(int(nbytes.value), dtype=torch.uint8)
    table = torch.empty(int(ntiles.value), 4, dtype=torch.int32)
    _abi.check(
        lib.wal_rvq_pack(ctypes.byref(geom), rows, ptrs, packed.data_ptr(), nbytes.value,
                         ctypes.cast(table.data_ptr(), ctypes.POINTER(ctypes.c_int32))),
        "wal_rvq_pack",
    )
    books = torch.stack(
        [torch.stack([c.detach().cpu().to(torch.float16) for c in g.codebooks]) for g in enc.groups]
    ).contiguous()
    rho = torch.cat([g.row_scale.detach().cpu().to(torch.float16).reshape(-1) for g in enc.groups]).contiguous()
    scales = None
    if any(g.stage_scales is not None for g in enc.groups):
        # groups without scales get 1.0 (fp32(c) * 1.0 == c: the same sum)
        scales = torch.stack([
            torch.ones(R, dtype=torch.float32) if g.stage_scales is None
            else g.stage_scales.detach().cpu().to(torch.float32).reshape(-1)[:R]
            for g in enc.groups]).contiguous()
        if scales.shape != (G, R):
            raise ValueError("stage_scales must hold one value per stage")
    return PackedArrays(geom, int(ntiles.value), packed, table, books, rho, scales)


def pack_routes(route: torch.Tensor, code: torch.Tensor, codebooks: torch.Tensor, row_scale: torch.Tensor,
                in_features: int) -> PackedArrays:
    """Pack a route-codebook weight (uint8 route and code per unit) through ``wal_route_pack``."""
    lib = _abi.load()
    G, C, d = (int(v) for v in codebooks.shape)
    if C != 256:
        raise ValueError("route-codebook packing expects 256 entries per routed codebook")
    N, B = (int(v) for v in route.shape)
    if tuple(code.shape) != (N, B) or B != -(-in_features // d):
        raise ValueError("route/code must be [out_features, ceil(in_features / d)]")
    geom = _geometry(N, in_features, d, 1, G * C, 1)
    rows = (ctypes.c_int64 * 1)(N)
    nbytes = ctypes.c_size_t(0)
    ntiles = ctypes.c_int64(0)
    _abi.check(lib.wal_rvq_packed_size(ctypes.byref(geom), rows, ctypes.byref(nbytes), ctypes.byref(ntiles)),
               "wal_rvq_packed_size")
    r = np.ascontiguousarray(route.detach().cpu().to(torch.uint8).numpy())
    c = np.ascontiguousarray(code.detach().cpu().to(torch.uint8).numpy())
    packed = torch.empty(int(nbytes.value), dtype=torch.uint8)
    table = torch.empty(int(ntiles.value), 4, dtype=torch.int32)
    _abi.check(
        lib.wal_route_pack(ctypes.byref(geom), r.ctypes.data, c.ctypes.data, packed.data_ptr(), nbytes.value,
                           ctypes.cast(table.data_ptr(), ctypes.POINTER(ctypes.c_int32))),
        "wal_route_pack",
    )
    books = codebooks.detach().cpu().to(torch.float16).reshape(1, 1, G * C, d).contiguous()
    rho = row_scale.detach().cpu().to(torch.float16).reshape(-1).contiguous()
    return PackedArrays(geom, int(ntiles.value), packed, table, books, rho)


# ---------------------------------------------------------------------------
# per-block corrections (reference src/runtime.py:389-412)
# ---------------------------------------------------------------------------
@dataclass
class CorrectionArrays:
    """Host tensors of ``wal_rvq_corrections`` for one linear (units = rows x blocks, groups concatenated)."""

    group_flags: torch.Tensor                # int32 [groups] of WAL_CORR_* bits
    residual_signs: Optional[torch.Tensor]   # int32 [N * blocks]
    residual_scale: Optional[torch.Tensor]   # fp16 [N * blocks]
    block_scale: Optional[torch.Tensor]      # fp16 [N * blocks]
    sign_matrix: Optional[torch.Tensor]      # fp32 [d, d]
    transform: Optional[torch.Tensor]        # fp32 [groups, d, d]
    transform_bias: Optional[torch.Tensor]   # fp32 [groups, d]


def hadamard_matrix(n: int) -> torch.Tensor:
    """Normalised Sylvester Hadamard matrix (the reference's ``_hadamard_matrix``, src/block_vq.py:10-22)."""
    if n < 1 or n & (n - 1):
        raise ValueError("hadamard transform requires power-of-two block_size")
    h = torch.ones(1, 1, dtype=torch.float32)
    while h.shape[0] < n:
        h = torch.cat((torch.cat((h, h), dim=1), torch.cat((h, -h), dim=1)), dim=0)
    return h / math.sqrt(float(n))


def rand_hadamard_matrix(n: int) -> torch.Tensor:
    """Row-permuted, row-signed Hadamard matrix from a fixed CPU generator (src/block_vq.py:25-35).

    The permutation and signs are drawn in the same order from a generator
    seeded with 0, so the matrix is the reference's, bit for bit.
    """
    base = hadamard_matrix(n)
    gen = torch.Generator(device="cpu").manual_seed(0)
    perm = torch.randperm(n, generator=gen)
    flip = torch.randint(0, 2, (n,), generator=gen, dtype=torch.int64) > 0
    signs = torch.where(flip, torch.ones(n), -torch.ones(n))
    return base[perm] * signs.unsqueeze(1)


def dct_matrix(n: int) -> torch.Tensor:
    """Orthonormal DCT-II matrix, rows = frequencies (src/block_vq.py:38-45)."""
    idx = torch.arange(n, dtype=torch.float32)
    mat = torch.cos(math.pi / float(n) * (idx + 0.5)[None, :] * idx[:, None])
    mat[0] *= math.sqrt(1.0 / float(n))
    if n > 1:
        mat[1:] *= math.sqrt(2.0 / float(n))
    return mat


def transform_matrix(kind: str, n: int) -> Optional[torch.Tensor]:
    """The fixed d x d matrix of a transform kind (None for none / polar / pca), src/block_vq.py:48-61."""
    if kind in ("none", "polar", "pca"):
        return None
    if kind == "dct":
        return dct_matrix(n)
    if kind == "hadamard":
        return hadamard_matrix(n)
    if kind == "rand_hadamard":
        return rand_hadamard_matrix(n)
    raise ValueError("transform_kind must be one of: none, dct, hadamard, rand_hadamard, polar, pca")


def pack_corrections(enc: GroupedBlockRVQEncoding) -> Optional[CorrectionArrays]:
    """Side arrays of the per-block corrections, or None when every group is plain."""
    if all(g.is_plain() for g in enc.groups):
        return None
    d = int(enc.groups[0].block_size)
    B = -(-int(enc.original_shape[1]) // d)
    G = len(enc.groups)
    flags = []
    signs, rscale, bscale = [], [], []
    mats = torch.zeros(G, d, d, dtype=torch.float32)
    tbias = torch.zeros(G, d, dtype=torch.float32)
    any_sign = any_bs = any_mat = any_bias = False
    for gi, g in enumerate(enc.groups):
        rows = int(g.original_shape[0])
        f = 0
        if g.residual_correction != "none" and g.residual_signs is not None and g.residual_scale is not None:
            words = g.residual_signs.detach().cpu().reshape(rows * B, -1)
            if words.shape[1] != 1:
                raise ValueError("sign residuals wider than 32 columns are not supported")
            signs.append(words[:, 0].to(torch.int32))
            rscale.append(g.residual_scale.detach().cpu().to(torch.float16).reshape(rows * B))
            f |= _abi.WAL_CORR_SIGN
            any_sign = True
        else:
            signs.append(torch.zeros(rows * B, dtype=torch.int32))
            rscale.append(torch.zeros(rows * B, dtype=torch.float16))
        if g.block_scale is not None:
            bscale.append(g.block_scale.detach().cpu().to(torch.float16).reshape(rows * B))
            f |= _abi.WAL_CORR_BLOCK_SCALE
            any_bs = True
        else:
            bscale.append(torch.ones(rows * B, dtype=torch.float16))
        if g.transform_kind == "polar":
            if d & (d - 1):
                raise ValueError("polar transform requires power-of-two block_size")
            f |= _abi.WAL_CORR_POLAR
        else:
            m = g.transform_matrix
            m = transform_matrix(g.transform_kind, d) if m is None else m.detach().cpu().to(torch.float32)
            if m is not None:
                mats[gi] = m.reshape(d, d)
                f |= _abi.WAL_CORR_MATRIX
                any_mat = True
        if g.transform_bias is not None:
            tbias[gi] = g.transform_bias.detach().cpu().to(torch.float32).reshape(d)
            f |= _abi.WAL_CORR_BIAS
            any_bias = True
        flags.append(f)
    return CorrectionArrays(
        group_flags=torch.tensor(flags, dtype=torch.int32),
        residual_signs=torch.cat(signs).contiguous() if any_sign else None,
        residual_scale=torch.cat(rscale).contiguous() if any_sign else None,
        block_scale=torch.cat(bscale).contiguous() if any_bs else None,
        sign_matrix=rand_hadamard_matrix(d).contiguous() if any_sign else None,
        transform=mats.contiguous() if any_mat else None,
        transform_bias=tbias.contiguous() if any_bias else None,
    )
