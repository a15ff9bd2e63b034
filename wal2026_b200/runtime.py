"""Drop-in runtime linear modules backed by the sm_100a CUDA library.

``PackedGroupedBlockRVQLinear`` keeps the constructor, attributes and forward
contract of the reference module of the same name (reference
``src/runtime.py:1175-1236`` and ``:1362-1507``): it takes a
``GroupedBlockRVQEncoding`` and an optional bias, exposes ``in_features``,
``out_features``, ``groups``, ``row_slices`` and ``reconstruct_weight``, and maps
``x[..., in_features]`` to ``y[..., out_features]`` in ``x.dtype``.  Every
``matmul_strategy`` the reference accepts is accepted here; they are
numerically interchangeable strategies in the reference, and this module always
runs its one fused kernel, which reproduces the default ``per_group`` path's
weight bit for bit.

There is no CPU path: the forward raises on CPU input, and the CUDA library
must be built (``python -m wal2026_b200.build``).
"""
from __future__ import annotations

import ctypes
import weakref
from typing import Optional

import torch
from torch import Tensor, nn

from . import _abi
from .block_vq import GroupedBlockRVQEncoding, single_group
from .packing import CorrectionArrays, PackedArrays, pack_corrections, pack_grouped, pack_routes

# the reference's accepted strategy names (src/runtime.py:1192)
MATMUL_STRATEGIES = frozenset({
    "per_group", "per_group_fast", "full_weight", "full_weight_fast", "full_weight_hot", "full_weight_hot_v2",
    "chunked_weight", "local_palette", "triton_hot_cold_persistent", "stage_local_hot_cold",
    "stage_local_hot_cold_b1", "stage_local_hot_cold_b2", "stage_local_hot_cold_b3", "stagewise_einsum",
    "triton_block_rvq", "stacked_matmul",
})

# strategies built on the reference's fast reconstruction
# (``reconstruct_weight_fast`` / ``_hot`` / ``_hot_v2``, src/runtime.py:568-798,
# and the hot-cold Triton paths whose CPU forms call them): stage tables
# rounded to the weight type and summed in it, and only the active stages of
# ``effective_stages_per_split`` (``_compute_active_stage_indices`` at
# src/runtime.py:588, :612, :663, :755, :930, :1045).  The others (per_group,
# full_weight, chunked_weight, local_palette, stagewise_einsum,
# triton_block_rvq, stacked_matmul) build the exact per_group weight from every
# stage whatever the setting.
FAST_STRATEGIES = frozenset({
    "per_group_fast", "full_weight_fast", "full_weight_hot", "full_weight_hot_v2", "triton_hot_cold_persistent",
    "stage_local_hot_cold", "stage_local_hot_cold_b1", "stage_local_hot_cold_b2", "stage_local_hot_cold_b3",
})

# token count from which the forward uses the tensor-core prefill GEMM
PREFILL_MIN_TOKENS = 128
# encodings with per-block corrections: the fused CUDA-core GEMV up to this many
# tokens, beyond it the corrected weight is materialised once for a library GEMM
CORRECTED_GEMV_MAX_TOKENS = 64

TARGET_LINEAR_SUFFIXES = (
    "self_attn.q_proj",
    "self_attn.k_proj",
    "self_attn.v_proj",
    "self_attn.o_proj",
    "mlp.gate_proj",
    "mlp.up_proj",
    "mlp.down_proj",
)


def _check_strategy_args(matmul_strategy, matmul_chunk_rows, local_palette_group_cols, hot_topk):
    """Same argument validation as reference ``src/runtime.py:1190-1211``."""
    if matmul_strategy == "triton_hot_cold_persistent" and local_palette_group_cols is None:
        local_palette_group_cols = 256
    if matmul_strategy not in MATMUL_STRATEGIES:
        raise ValueError(f"unsupported matmul_strategy: {matmul_strategy}")
    if matmul_strategy == "chunked_weight" and (matmul_chunk_rows is None or int(matmul_chunk_rows) <= 0):
        raise ValueError("chunked_weight requires a positive matmul_chunk_rows")
    if matmul_strategy in {"local_palette", "triton_hot_cold_persistent"} and (
        local_palette_group_cols is None or int(local_palette_group_cols) <= 0
    ):
        raise ValueError(f"{matmul_strategy} requires a positive local_palette_group_cols")
    needs_topk = {"full_weight_hot", "full_weight_hot_v2", "triton_hot_cold_persistent", "stage_local_hot_cold",
                  "stage_local_hot_cold_b1", "stage_local_hot_cold_b2", "stage_local_hot_cold_b3"}
    if matmul_strategy in needs_topk and (hot_topk is None or int(hot_topk) <= 0):
        raise ValueError(f"{matmul_strategy} requires a positive hot_topk")
    return local_palette_group_cols


class PackedBlockRVQGroup(nn.Module):
    """One row group of a packed linear (reference ``src/runtime.py:248``).

    The ids of every group live in the parent's single packed stream; a group
    keeps its shape attributes, its codebooks and row scales (small) and
    reaches the parent through a weak reference for ``reconstruct_weight``.
    """

    def __init__(self, parent: "PackedGroupedBlockRVQLinear", row0: int, row1: int, *, block_size: int,
                 in_features: int, num_stages: int, enc=None) -> None:
        super().__init__()
        self.block_size = int(block_size)
        self.in_features = int(in_features)
        self.out_features = int(row1 - row0)
        self.padded_cols = -(-self.in_features // self.block_size) * self.block_size
        self.num_stages = int(num_stages)
        self.product_splits = 1 if enc is None else int(enc.product_splits)
        self.stages_per_split = (self.num_stages,) if enc is None else tuple(int(x) for x in enc.stages_per_split)
        self.transform_kind = "none" if enc is None else enc.transform_kind
        self.residual_correction = "none" if enc is None else enc.residual_correction
        self.row0, self.row1 = int(row0), int(row1)
        self._parent = weakref.ref(parent)
        # variable-stage decoding (reference src/runtime.py:320-323, :352-377):
        # keep the first k stages of every product split
        self.effective_stages_per_split: int = max(self.stages_per_split) if self.stages_per_split \
            else self.num_stages
        self._active_stage_indices: Optional[tuple[int, ...]] = None

    def _compute_active_stage_indices(self) -> tuple[int, ...]:
        """Stage indices summed under ``effective_stages_per_split`` (reference ``src/runtime.py:352-372``).

        Stages are stored split-major (split 0's stages, then split 1's, ...);
        the first ``k`` stages of every split are kept, at least one stage in all.
        """
        if self._active_stage_indices is not None:
            return self._active_stage_indices
        keep = max(1, int(self.effective_stages_per_split))
        idxs: list[int] = []
        offset = 0
        for count in self.stages_per_split:
            idxs.extend(offset + j for j in range(min(keep, int(count))))
            offset += int(count)
        self._active_stage_indices = tuple(idxs) if idxs else (0,)
        return self._active_stage_indices

    def set_effective_stages_per_split(self, k: int) -> None:
        """Set the per-split active stage count (reference ``src/runtime.py:374-377``)."""
        self.effective_stages_per_split = int(k)
        self._active_stage_indices = None

    def reconstruct_weight(self, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        parent = self._parent()
        if parent is None:
            raise RuntimeError("group outlived its packed linear")
        return parent.reconstruct_weight(out_dtype)[self.row0:self.row1]

    def reconstruct_weight_fast(self, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        parent = self._parent()
        if parent is None:
            raise RuntimeError("group outlived its packed linear")
        return parent.reconstruct_weight_fast(out_dtype)[self.row0:self.row1]


class PackedGroupedBlockRVQLinear(nn.Module):
    """Block-RVQ linear with packed ids and the fused CUDA decode GEMV."""

    def __init__(
        self,
        enc: GroupedBlockRVQEncoding,
        bias: Optional[Tensor] = None,
        *,
        matmul_strategy: str = "per_group",
        matmul_chunk_rows: Optional[int] = None,
        local_palette_group_cols: Optional[int] = None,
        hot_topk: Optional[int] = None,
        hot_score_mode: str = "row_scale_norm",
        hot_min_stage_share: float = 0.0,
        hot_score_threshold_ratio: float = 0.0,
        _packed: Optional[PackedArrays] = None,
    ) -> None:
        super().__init__()
        local_palette_group_cols = _check_strategy_args(matmul_strategy, matmul_chunk_rows,
                                                        local_palette_group_cols, hot_topk)
        if not isinstance(enc, GroupedBlockRVQEncoding):
            enc = single_group(enc)
        self.in_features = int(enc.original_shape[1])
        self.out_features = int(enc.original_shape[0])
        self.row_slices = tuple(tuple(int(v) for v in s) for s in enc.row_slices)
        self.matmul_strategy = matmul_strategy
        self.matmul_chunk_rows = None if matmul_chunk_rows is None else int(matmul_chunk_rows)
        self.local_palette_group_cols = None if local_palette_group_cols is None else int(local_palette_group_cols)
        self.hot_topk = None if hot_topk is None else int(hot_topk)
        self.hot_score_mode = hot_score_mode
        self.hot_min_stage_share = float(hot_min_stage_share)
        self.hot_score_threshold_ratio = float(hot_score_threshold_ratio)
        packed = _packed if _packed is not None else pack_grouped(enc, allow_corrections=True)
        self._set_packed(packed)
        self._set_corrections(pack_corrections(enc))
        self.groups = nn.ModuleList(
            PackedBlockRVQGroup(self, r0, r1, block_size=g.block_size, in_features=self.in_features,
                                num_stages=len(g.stage_ids), enc=g)
            for g, (r0, r1) in zip(enc.groups, self.row_slices)
        )
        if bias is not None:
            self.register_buffer("bias", bias.detach().to(torch.bfloat16).reshape(-1).contiguous())
        else:
            self.bias = None
        self._layer_cache: tuple | None = None

    def _set_packed(self, packed: PackedArrays) -> None:
        g = packed.geometry
        self.block_size = int(g.block_size)
        self.num_stages = int(g.num_stages)
        self.num_entries = int(g.num_entries)
        self.num_groups = int(g.num_groups)
        self.num_tiles = int(packed.num_tiles)
        self.register_buffer("packed_ids", packed.packed_ids)
        self.register_buffer("tile_table", packed.tile_table)
        self.register_buffer("codebooks", packed.codebooks)
        self.register_buffer("row_scale", packed.row_scale)
        if packed.stage_scales is not None:
            self.register_buffer("stage_scales", packed.stage_scales.to(torch.float32).contiguous())
        else:
            self.stage_scales = None

    CORRECTION_BUFFERS = ("corr_flags", "corr_signs", "corr_rscale", "corr_bscale", "corr_sign_matrix",
                          "corr_transform", "corr_tbias")

    def _set_corrections(self, corr: Optional[CorrectionArrays]) -> None:
        """Register the per-block correction arrays (reference ``src/runtime.py:266-290`` buffers) or mark none."""
        self.has_corrections = corr is not None
        values = (None,) * len(self.CORRECTION_BUFFERS) if corr is None else (
            corr.group_flags, corr.residual_signs, corr.residual_scale, corr.block_scale, corr.sign_matrix,
            corr.transform, corr.transform_bias)
        for name, value in zip(self.CORRECTION_BUFFERS, values):
            if value is None:
                setattr(self, name, None)
            else:
                self.register_buffer(name, value)

    def corrections_struct(self) -> _abi.Corrections:
        """The ``wal_rvq_corrections`` descriptor of this module's correction buffers."""
        ptrs = [None if getattr(self, n) is None else getattr(self, n).data_ptr() for n in self.CORRECTION_BUFFERS]
        return _abi.Corrections(*ptrs)

    @classmethod
    def random(
        cls,
        group_rows: list[int],
        in_features: int,
        *,
        block_size: int = 8,
        num_stages: int = 2,
        entries: int = 256,
        stage_std: tuple[float, ...] = (0.02, 0.005),
        generator: Optional[torch.Generator] = None,
        device: torch.device | str = "cuda",
        bias: Optional[Tensor] = None,
    ) -> "PackedGroupedBlockRVQLinear":
        """A packed linear with seeded random ids, codebooks and row scales, built on ``device``.

        For benchmark stacks whose weights are random by definition: uniform ids
        are written straight into the packed stream (any permutation of
        uniform ids is uniform), codebooks are N(0, stage_std[s]) fp16 and row
        scales U(0.5, 1.5) fp16, so no dense weight and no host-side encoding
        is ever materialised.  The result is a regular packed module (it
        round-trips through ``unpack_ids``).
        """
        if entries > 256:
            raise ValueError("random() builds 1-byte ids (<= 256 entries)")
        device = torch.device(device)
        gen = generator
        d, R, K = int(block_size), int(num_stages), int(in_features)
        N = int(sum(group_rows))
        blocks = -(-K // d)
        chunks = -(-blocks // 16)
        tiles = [-(-int(n) // 16) for n in group_rows]
        T = sum(tiles)
        nbytes = T * chunks * R * 256
        if entries == 256:
            packed = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=device, generator=gen)
        else:
            packed = torch.randint(0, entries, (nbytes,), dtype=torch.uint8, device=device, generator=gen)
        table = []
        row0 = 0
        for g, (n, t) in enumerate(zip(group_rows, tiles)):
            for lt in range(t):
                table.append([g, row0 + 16 * lt, min(16, int(n) - 16 * lt), 0])
            row0 += int(n)
        books = torch.empty((len(group_rows), R, entries, d), device=device, dtype=torch.float32)
        for s in range(R):
            std = stage_std[s] if s < len(stage_std) else stage_std[-1]
            books[:, s].normal_(0.0, std, generator=gen)
        rho = torch.rand((N,), device=device, generator=gen) + 0.5
        geom = _abi.Geometry(out_features=N, in_features=K, block_size=d, num_stages=R, num_entries=entries,
                             num_groups=len(group_rows))
        arrays = PackedArrays(geom, T, packed, torch.tensor(table, dtype=torch.int32, device=device),
                              books.to(torch.float16).contiguous(), rho.to(torch.float16).contiguous())
        return cls.from_packed(arrays, group_rows, bias=bias)

    @classmethod
    def from_packed(cls, arrays: PackedArrays, group_rows: list[int],
                    bias: Optional[Tensor] = None) -> "PackedGroupedBlockRVQLinear":
        """A module over already packed arrays (e.g. a tensor-parallel shard of another module)."""
        g = arrays.geometry
        K, N, d, R = int(g.in_features), int(g.out_features), int(g.block_size), int(g.num_stages)
        if sum(int(n) for n in group_rows) != N or len(group_rows) != int(g.num_groups):
            raise ValueError("group_rows do not match the packed geometry")
        obj = cls.__new__(cls)
        nn.Module.__init__(obj)
        obj.in_features, obj.out_features = K, N
        slices, r = [], 0
        for n in group_rows:
            slices.append((r, r + int(n)))
            r += int(n)
        obj.row_slices = tuple(slices)
        obj.matmul_strategy = "per_group"
        obj.matmul_chunk_rows = obj.local_palette_group_cols = obj.hot_topk = None
        obj.hot_score_mode, obj.hot_min_stage_share, obj.hot_score_threshold_ratio = "row_scale_norm", 0.0, 0.0
        obj._set_packed(arrays)
        obj._set_corrections(None)
        obj.groups = nn.ModuleList(PackedBlockRVQGroup(obj, r0, r1, block_size=d, in_features=K, num_stages=R)
                                   for r0, r1 in obj.row_slices)
        if bias is not None:
            obj.register_buffer("bias", bias.detach().to(device=arrays.packed_ids.device,
                                                         dtype=torch.bfloat16).reshape(-1).contiguous())
        else:
            obj.bias = None
        obj._layer_cache = None
        return obj

    def packed_arrays(self) -> PackedArrays:
        """This module's packed buffers (shared, not copied)."""
        geom = _abi.Geometry(out_features=self.out_features, in_features=self.in_features,
                             block_size=self.block_size, num_stages=self.num_stages,
                             num_entries=self.num_entries, num_groups=self.num_groups)
        return PackedArrays(geom, self.num_tiles, self.packed_ids, self.tile_table, self.codebooks, self.row_scale,
                            self.stage_scales)

    def group_rows(self) -> list[int]:
        return [r1 - r0 for r0, r1 in self.row_slices]

    # -- C ABI plumbing -----------------------------------------------------
    def _active_stages(self) -> Optional[tuple[tuple[int, ...], ...]]:
        """Per-group active stage indices when this strategy drops stages, else None (all stages).

        Encodings with per-block corrections always sum every stage: the
        reference's fast reconstruction falls back to the full one for them
        (``supports_fast_reconstruct``, ``src/runtime.py:416-429``).
        """
        if self.matmul_strategy not in FAST_STRATEGIES or self.has_corrections:
            return None
        active = tuple(g._compute_active_stage_indices() for g in self.groups)
        full = tuple(range(self.num_stages))
        return None if all(a == full for a in active) else active

    def _stage_view(self, active: tuple[tuple[int, ...], ...]) -> tuple:
        """Packed stream, codebooks and stage scales holding only the union of the active stages.

        Cut from this module's device buffers (the packed stream keeps whole
        16-byte stage vectors, so the cut is a selection of vectors per
        chunk): the GEMV then streams only the active stages' ids.  A stage
        of the union that a group does not keep gets an all-zero codebook in
        that group; adding +0.0 to the fp32 stage sum changes no bit (the sum
        starts from +0.0, so it is never -0.0).  Cached per active set.
        """
        key = (active, self.packed_ids.data_ptr(), self.codebooks.data_ptr())
        cache = getattr(self, "_stage_cache", None)
        if cache is not None and cache[0] == key:
            return cache[1]
        union = sorted(set().union(*active))
        idw = 1 if self.num_entries <= 256 else 2
        blocks = -(-self.in_features // self.block_size)
        chunks = -(-blocks // 16)
        V = self.num_stages * idw
        vec = torch.tensor([s * idw + h for s in union for h in range(idw)], device=self.packed_ids.device)
        packed = self.packed_ids.view(self.num_tiles * chunks, V, 256).index_select(1, vec).reshape(-1).contiguous()
        books = self.codebooks[:, union].clone()
        for g, act in enumerate(active):
            for j, st in enumerate(union):
                if st not in act:
                    books[g, j].zero_()
        scales = None if self.stage_scales is None else self.stage_scales[:, union].contiguous()
        view = (len(union), packed, books.contiguous(), scales)
        self._stage_cache = (key, view)
        return view

    def sum_mode(self) -> int:
        """``WAL_SUM_FAST`` for the strategies built on the reference's fast reconstruction, else exact."""
        fast = self.matmul_strategy in FAST_STRATEGIES and not self.has_corrections
        return _abi.WAL_SUM_FAST if fast else _abi.WAL_SUM_EXACT

    def layer_struct(self, stages: Optional[tuple[tuple[int, ...], ...]] = None,
                     sum_mode: int = _abi.WAL_SUM_EXACT) -> _abi.Layer:
        """The ``wal_rvq_layer`` descriptor of this module's current device buffers.

        ``stages``: per-group active stage indices (``_active_stages()``); the
        descriptor then points at the stage view holding only those stages.
        ``sum_mode``: how stage values become a weight (``WAL_SUM_*``).
        """
        R, packed, books, scales = self.num_stages, self.packed_ids, self.codebooks, self.stage_scales
        if stages is not None:
            R, packed, books, scales = self._stage_view(stages)
        key = (R, packed.data_ptr(), self.tile_table.data_ptr(), books.data_ptr(),
               self.row_scale.data_ptr(), None if self.bias is None else self.bias.data_ptr(),
               None if scales is None else scales.data_ptr(), int(sum_mode))
        if self._layer_cache is not None and self._layer_cache[0] == key:
            return self._layer_cache[1]
        geom = _abi.Geometry(out_features=self.out_features, in_features=self.in_features,
                             block_size=self.block_size, num_stages=R,
                             num_entries=self.num_entries, num_groups=self.num_groups)
        rows = [r1 - r0 for r0, r1 in self.row_slices]
        self._group_rows = (ctypes.c_int64 * len(rows))(*rows)  # kept alive with the descriptor
        layer = _abi.Layer(geom=geom, num_tiles=self.num_tiles, packed_ids=key[1], tile_table=key[2],
                           codebooks=key[3], row_scale=key[4], bias=key[5],
                           group_rows=ctypes.cast(self._group_rows, ctypes.POINTER(ctypes.c_int64)),
                           stage_scales=key[6], sum_mode=key[7])
        self._layer_cache = (key, layer)
        return layer

    def _require_cuda(self, x: Tensor) -> None:
        if not x.is_cuda:
            raise ValueError("PackedGroupedBlockRVQLinear runs on CUDA only (no CPU path); move the input "
                             "and the module to a CUDA device")
        if self.packed_ids.device != x.device:
            raise ValueError(f"input on {x.device} but module buffers on {self.packed_ids.device}")

    # -- public API ---------------------------------------------------------
    def forward(self, x: Tensor) -> Tensor:
        """y = x @ w^T (+ bias) in ``x.dtype`` (bf16, fp16 or fp32), as the reference forward.

        The weight is decoded in ``x.dtype`` with the reference's roundings
        for this strategy (``reconstruct_weight`` for per_group and the other
        exact strategies, ``reconstruct_weight_fast`` for the fast ones) and
        never materialised; products accumulate in fp32.
        """
        self._require_cuda(x)
        if x.dtype not in _abi.DTYPE_CODE:
            raise ValueError(f"PackedGroupedBlockRVQLinear supports bfloat16, float16 and float32 activations, "
                             f"got {x.dtype}")
        orig = x.shape
        if orig[-1] != self.in_features:
            raise ValueError(f"Feature mismatch: {orig[-1]} != {self.in_features}")
        x2 = x.reshape(-1, self.in_features)
        align = 4 if x.dtype == torch.float32 else 8  # elements per 16 bytes
        if x2.stride(-1) != 1 or x2.stride(0) % align != 0 or x2.data_ptr() % 16 != 0:
            if self.in_features % align == 0:
                x2 = x2.contiguous()
            else:  # pad rows so every row starts 16-byte aligned
                xp = torch.zeros((x2.shape[0], -(-self.in_features // align) * align), device=x.device,
                                 dtype=x.dtype)
                xp[:, :self.in_features] = x2
                x2 = xp
        M = x2.shape[0]
        if self.has_corrections and M > CORRECTED_GEMV_MAX_TOKENS:
            # the corrected weight once, then a library GEMM (the reference's own per_group scheme)
            w = self.reconstruct_weight(x.dtype)
            bias = None if self.bias is None else self.bias.to(x.dtype)
            return torch.nn.functional.linear(x2, w, bias).reshape(*orig[:-1], self.out_features)
        y = torch.empty((M, self.out_features), device=x.device, dtype=x.dtype)
        if M >= PREFILL_MIN_TOKENS and x.dtype != torch.float32 and self.gemm_into(x2, y):
            pass
        elif M > 0:
            self.gemv_into(x2, y)
        return y.reshape(*orig[:-1], self.out_features)

    def gemm_into(self, x2: Tensor, y: Tensor, status: Optional[Tensor] = None) -> bool:
        """Prefill GEMM on the tcgen05 path; False when this layer's format is not covered by it."""
        if self.has_corrections:
            return False
        lib = _abi.load()
        layer = self.layer_struct(self._active_stages(), self.sum_mode())
        with torch.cuda.device(x2.device):
            st = lib.wal_rvq_gemm_typed(ctypes.byref(layer), x2.data_ptr(), _abi.DTYPE_CODE[x2.dtype], x2.shape[0],
                                        x2.stride(0), y.data_ptr(), y.stride(0), _abi.DTYPE_CODE[y.dtype],
                                        None if status is None else status.data_ptr(), _abi.stream_handle(x2.device))
        if st == _abi.WAL_ERR_UNSUPPORTED:
            return False
        _abi.check(st, "wal_rvq_gemm")
        return True

    def gemv_into(self, x2: Tensor, y: Tensor, *, warps_per_tile: int = 0, num_ctas: int = 0) -> None:
        """y[M, N] <- x2[M, K] @ w^T (+ bias) through ``wal_rvq_gemv_typed`` on the current stream."""
        lib = _abi.load()
        layer = self.layer_struct(self._active_stages(), self.sum_mode())
        if self.has_corrections:
            corr = self.corrections_struct()
            with torch.cuda.device(x2.device):
                st = lib.wal_rvq_gemv_corrected(ctypes.byref(layer), ctypes.byref(corr), x2.data_ptr(),
                                                _abi.DTYPE_CODE[x2.dtype], x2.shape[0], x2.stride(0), y.data_ptr(),
                                                y.stride(0), _abi.DTYPE_CODE[y.dtype], _abi.stream_handle(x2.device))
            _abi.check(st, "wal_rvq_gemv_corrected")
            return
        # decode-sized calls are short (a few us on the GPU), so the host path
        # avoids a device switch when the input's device is already current
        dev = x2.device
        args = (ctypes.byref(layer), x2.data_ptr(), _abi.DTYPE_CODE[x2.dtype], x2.shape[0], x2.stride(0),
                y.data_ptr(), y.stride(0), _abi.DTYPE_CODE[y.dtype], warps_per_tile, num_ctas)
        if dev.index == torch.cuda.current_device():
            st = lib.wal_rvq_gemv_typed(*args, _abi.stream_handle(dev))
        else:
            with torch.cuda.device(dev):
                st = lib.wal_rvq_gemv_typed(*args, _abi.stream_handle(dev))
        if st:
            _abi.check(st, "wal_rvq_gemv")

    def reconstruct_weight(self, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        """The weight in ``out_dtype`` (bf16, fp16 or fp32), bit-identical to the reference's
        ``reconstruct_weight(out_dtype)`` (every stage, exact sum; ``src/runtime.py:1234-1236``)."""
        return self._dequant(out_dtype, None, _abi.WAL_SUM_EXACT)

    def reconstruct_weight_fast(self, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        """The weight of the reference's ``reconstruct_weight_fast(out_dtype)`` (``src/runtime.py:1238-1240``):
        the active stages of ``effective_stages_per_split``, each rounded to ``out_dtype`` and summed in it."""
        if self.has_corrections:  # the reference falls back to the full reconstruction
            return self.reconstruct_weight(out_dtype)
        active = tuple(g._compute_active_stage_indices() for g in self.groups)
        full = tuple(range(self.num_stages))
        return self._dequant(out_dtype, None if all(a == full for a in active) else active, _abi.WAL_SUM_FAST)

    def _dequant(self, out_dtype: torch.dtype, stages, sum_mode: int) -> Tensor:
        if out_dtype not in _abi.DTYPE_CODE:
            raise ValueError(f"reconstruct_weight supports bfloat16, float16 and float32, got {out_dtype}")
        dev = self.packed_ids.device
        if dev.type != "cuda":
            raise ValueError("reconstruct_weight runs on CUDA only; move the module to a CUDA device")
        w = torch.empty((self.out_features, self.in_features), device=dev, dtype=out_dtype)
        lib = _abi.load()
        if self.has_corrections:
            corr = self.corrections_struct()
            with torch.cuda.device(dev):
                st = lib.wal_rvq_dequant_corrected(ctypes.byref(self.layer_struct()), ctypes.byref(corr), w.data_ptr(),
                                                   w.stride(0), _abi.DTYPE_CODE[out_dtype], _abi.stream_handle(dev))
            _abi.check(st, "wal_rvq_dequant_corrected")
            return w
        with torch.cuda.device(dev):
            st = lib.wal_rvq_dequant_typed(ctypes.byref(self.layer_struct(stages, sum_mode)), w.data_ptr(),
                                           w.stride(0), _abi.DTYPE_CODE[out_dtype], _abi.stream_handle(dev))
        _abi.check(st, "wal_rvq_dequant")
        return w

    def unpack_ids(self) -> Tensor:
        """Packed stream read back on the device: ids [R, N, blocks] (uint8 or int16)."""
        dev = self.packed_ids.device
        if dev.type != "cuda":
            raise ValueError("unpack_ids runs on CUDA only")
        blocks = -(-self.in_features // self.block_size)
        dtype = torch.uint8 if self.num_entries <= 256 else torch.int16
        out = torch.empty((self.num_stages, self.out_features, blocks), device=dev, dtype=dtype)
        lib = _abi.load()
        with torch.cuda.device(dev):
            st = lib.wal_rvq_unpack_ids(ctypes.byref(self.layer_struct()), out.data_ptr(), _abi.stream_handle(dev))
        _abi.check(st, "wal_rvq_unpack_ids")
        return out

    def compressed_bytes(self) -> int:
        """Bytes a decode GEMV must read for the weight: ids + codebooks + row scales (+ bias)."""
        blocks = -(-self.in_features // self.block_size)
        idw = 1 if self.num_entries <= 256 else 2
        total = self.out_features * blocks * self.num_stages * idw
        total += self.codebooks.numel() * 2 + self.out_features * 2
        if self.bias is not None:
            total += self.out_features * 2
        return total

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, block_size={self.block_size}, "
                f"num_stages={self.num_stages}, entries={self.num_entries}, groups={self.num_groups}, "
                f"matmul_strategy={self.matmul_strategy}")


class RouteCodebookLinear(PackedGroupedBlockRVQLinear):
    """Route-codebook linear: per unit a route over G codebooks plus a code.

    No module of this name exists in the reference; the format is the
    one-stage special case of its Block-RVQ path (id = route * 256 + code into
    the flattened ``[G * 256, d]`` codebook), so this class is a
    ``PackedGroupedBlockRVQLinear`` whose ids are packed from route/code arrays.
    """

    @classmethod
    def from_routes(cls, route: Tensor, code: Tensor, codebooks: Tensor, row_scale: Tensor,
                    bias: Optional[Tensor] = None, *, in_features: int, **kwargs) -> "RouteCodebookLinear":
        """Build from uint8 ``route``/``code`` ``[N, blocks]``, fp16 ``codebooks`` ``[G, 256, d]``, fp16 ``row_scale``."""
        from .block_vq import route_code_encoding

        packed = pack_routes(route, code, codebooks, row_scale, in_features)
        enc = single_group(route_code_encoding(route, code, codebooks, row_scale, in_features=in_features))
        return cls(enc, bias, _packed=packed, **kwargs)


def _set_submodule(root: nn.Module, path: str, module: nn.Module) -> None:
    parent = root
    parts = path.split(".")
    for part in parts[:-1]:
        parent = getattr(parent, part)
    setattr(parent, parts[-1], module)


@torch.no_grad()
def replace_with_preencoded_packed_block_rvq(
    model: nn.Module,
    encodings_by_name: dict[str, GroupedBlockRVQEncoding],
    *,
    matmul_strategy: str = "per_group",
    device: Optional[torch.device] = None,
    **strategy_kwargs,
) -> list[dict[str, object]]:
    """Swap named ``nn.Linear`` modules for packed modules built from encodings.

    Mirrors reference ``src/runtime.py:2145-2200``: every ``nn.Linear`` whose
    name is a key of ``encodings_by_name`` is replaced in place; the original
    weight is released.  Returns one stats dict per replaced layer.
    """
    stats = []
    for name, module in list(model.named_modules()):
        if name not in encodings_by_name or not isinstance(module, nn.Linear):
            continue
        enc = encodings_by_name[name]
        target = device if device is not None else module.weight.device
        packed = PackedGroupedBlockRVQLinear(enc, module.bias, matmul_strategy=matmul_strategy,
                                             **strategy_kwargs).to(target)
        _set_submodule(model, name, packed)
        stats.append({
            "name": name,
            "tensor_name": f"{name}.weight",
            "runtime_decision": "preencoded_packed_block_rvq",
            "matmul_strategy": matmul_strategy,
            "storage_bytes": int(enc.storage_bytes()),
            "bits_per_weight": float(enc.bits_per_weight()),
        })
    return stats


# ---------------------------------------------------------------------------
# variable-stage decoding helpers (reference src/runtime.py:2274-2327)
# ---------------------------------------------------------------------------
def set_global_effective_stages(model: nn.Module, stages: int) -> int:
    """Set ``effective_stages_per_split`` on every ``PackedBlockRVQGroup``; returns the groups updated."""
    n = 0
    for module in model.modules():
        if isinstance(module, PackedBlockRVQGroup):
            module.set_effective_stages_per_split(int(stages))
            n += 1
    return n


def set_effective_stages_by_name(model: nn.Module, attn_stages: Optional[int],
                                 mlp_stages: Optional[int]) -> dict[str, int]:
    """Per-role stage cap: ``.self_attn.`` linears get ``attn_stages``, ``.mlp.`` ones ``mlp_stages``."""
    counts = {"attn": 0, "mlp": 0, "other": 0}
    for name, module in model.named_modules():
        if not isinstance(module, PackedGroupedBlockRVQLinear):
            continue
        bucket = "attn" if ".self_attn." in name else ("mlp" if ".mlp." in name else "other")
        target = attn_stages if bucket == "attn" else (mlp_stages if bucket == "mlp" else None)
        if target is None:
            continue
        for sub in module.modules():
            if isinstance(sub, PackedBlockRVQGroup):
                sub.set_effective_stages_per_split(int(target))
        counts[bucket] += 1
    return counts


def set_effective_stages_from_map(model: nn.Module, name_to_k: dict[str, int]) -> int:
    """Per-layer stage cap from ``{layer name: k}``; returns the layers updated (unknown names skipped)."""
    updated = 0
    for name, module in model.named_modules():
        if not isinstance(module, PackedGroupedBlockRVQLinear) or name not in name_to_k:
            continue
        k = int(name_to_k[name])
        for sub in module.modules():
            if isinstance(sub, PackedBlockRVQGroup):
                sub.set_effective_stages_per_split(k)
        updated += 1
    return updated
