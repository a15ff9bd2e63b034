"""Block-RVQ encoding containers, field-compatible with the reference.

The reference stores an encoded weight matrix as a dataclass of per-stage id
tensors, per-stage fp16 codebooks and a per-row fp16 scale
(reference ``src/block_vq.py:230-257`` for ``BlockRVQEncoding`` and
``src/block_vq.py:316-320`` for ``GroupedBlockRVQEncoding``).  These classes
keep the same field names and meanings so that an encoding produced or saved by
the reference can be handed to this package unchanged (``encoding_io`` reads the
reference's on-disk map).  Only containers live here: the offline k-means
encoder is out of scope for the runtime build.

Weight semantics (reference ``src/block_vq.py:259-289``, restated):

* the matrix has ``rows`` output rows and ``original_shape[1]`` input columns,
  padded on the right to ``padded_cols = blocks * block_size``;
* unit ``(row, block)`` of stage ``s`` selects row ``stage_ids[s][row, block]``
  of ``codebooks[s]`` (shape ``[entries, block_size]``, fp16);
* the dequantised weight is ``bf16(bf16(sum_s fp32(entry_s)) * bf16(row_scale))``
  for a bf16 forward (two bf16 roundings, fp32 stage sum, stage order 0..R-1).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch
from torch import Tensor


@dataclass
class BlockRVQEncoding:
    """One row group of a Block-RVQ weight (reference ``src/block_vq.py:230``)."""

    stage_ids: tuple[Tensor, ...]
    codebooks: tuple[Tensor, ...]
    stage_value_dims: tuple[int, ...]
    stages_per_split: tuple[int, ...]
    stage_scales: Optional[Tensor]
    residual_correction: str
    residual_signs: Optional[Tensor]
    residual_scale: Optional[Tensor]
    row_scale: Tensor
    block_scale: Optional[Tensor]
    transform_kind: str
    transform_matrix: Optional[Tensor]
    transform_bias: Optional[Tensor]
    product_splits: int
    original_shape: tuple[int, int]
    padded_cols: int
    block_size: int
    sample_rel_mse: float = 0.0

    @property
    def num_stages(self) -> int:
        return len(self.codebooks)

    @property
    def stage_shape(self) -> tuple[int, int]:
        return tuple(int(v) for v in self.stage_ids[0].shape)

    def is_plain(self) -> bool:
        """True when the encoding uses none of the per-block corrections.

        Plain encodings (the sum of stages, with optional per-stage scales:
        each stage value ``fp32(c) * scale`` before the sum, reference
        ``src/block_vq.py:264-268``) run on the tensor-core decode kernels;
        block scales, sign residuals and transforms (reference
        ``src/runtime.py:389-412``) run on the corrected-decode kernels.
        """
        return (
            self.block_scale is None
            and self.transform_kind == "none"
            and self.transform_matrix is None
            and self.transform_bias is None
            and (self.residual_correction == "none" or self.residual_signs is None)
        )

    def storage_bytes(self) -> int:
        """Bytes of the encoded form, counted like reference ``src/block_vq.py:291-309``."""
        total = 0
        for ids, codebook, value_dim in zip(self.stage_ids, self.codebooks, self.stage_value_dims):
            entries = int(codebook.shape[0])
            id_bytes = 1 if entries <= 256 else (2 if entries <= 65536 else 4)
            total += ids.numel() * id_bytes
            total += entries * int(value_dim) * 2
        for extra in (self.stage_scales, self.residual_signs, self.residual_scale, self.block_scale,
                      self.transform_matrix, self.transform_bias):
            if extra is not None:
                total += extra.numel() * extra.element_size()
        total += self.row_scale.numel() * 2
        return total

    def bits_per_weight(self) -> float:
        rows, cols = self.original_shape
        return 8.0 * self.storage_bytes() / max(rows * cols, 1)


@dataclass
class GroupedBlockRVQEncoding:
    """Row-sliced groups, each with its own codebooks (reference ``src/block_vq.py:316``)."""

    groups: tuple[BlockRVQEncoding, ...]
    row_slices: tuple[tuple[int, int], ...]
    original_shape: tuple[int, int]

    def storage_bytes(self) -> int:
        return sum(g.storage_bytes() for g in self.groups)

    def bits_per_weight(self) -> float:
        rows, cols = self.original_shape
        return 8.0 * self.storage_bytes() / max(rows * cols, 1)


def make_plain_encoding(
    stage_ids: list[Tensor] | tuple[Tensor, ...],
    codebooks: list[Tensor] | tuple[Tensor, ...],
    row_scale: Tensor,
    *,
    in_features: int,
    block_size: int,
) -> BlockRVQEncoding:
    """Build a plain (correction-free) encoding from ids, codebooks and row scales.

    ``stage_ids[s]`` is ``[rows, blocks]`` (uint8 for <=256 entries, int16 for
    larger codebooks, matching reference ``src/block_vq.py:159-164``),
    ``codebooks[s]`` is ``[entries, block_size]`` fp16 and ``row_scale`` is
    ``[rows, 1]`` fp16.
    """
    rows, blocks = (int(v) for v in stage_ids[0].shape)
    if blocks * block_size < in_features:
        raise ValueError("blocks * block_size must cover in_features")
    return BlockRVQEncoding(
        stage_ids=tuple(t.contiguous() for t in stage_ids),
        codebooks=tuple(c.to(torch.float16).contiguous() for c in codebooks),
        stage_value_dims=tuple(block_size for _ in codebooks),
        stages_per_split=(len(codebooks),),
        stage_scales=None,
        residual_correction="none",
        residual_signs=None,
        residual_scale=None,
        row_scale=row_scale.to(torch.float16).reshape(rows, 1).contiguous(),
        block_scale=None,
        transform_kind="none",
        transform_matrix=None,
        transform_bias=None,
        product_splits=1,
        original_shape=(rows, int(in_features)),
        padded_cols=blocks * block_size,
        block_size=int(block_size),
        sample_rel_mse=0.0,
    )


def single_group(enc: BlockRVQEncoding) -> GroupedBlockRVQEncoding:
    """Wrap one encoding as a one-group grouped encoding covering all rows."""
    rows = int(enc.original_shape[0])
    return GroupedBlockRVQEncoding(groups=(enc,), row_slices=((0, rows),), original_shape=enc.original_shape)


def route_code_encoding(
    route: Tensor,
    code: Tensor,
    codebooks: Tensor,
    row_scale: Tensor,
    *,
    in_features: int,
) -> BlockRVQEncoding:
    """Express a route-codebook weight as a single-stage Block-RVQ encoding.

    Each unit carries a route id over ``G`` codebooks and a code into the
    selected codebook (``codebooks`` is ``[G, entries, d]`` fp16).  This is
    exactly a one-stage encoding with id ``route * entries + code`` into the
    flattened ``[G * entries, d]`` codebook, which is how the reference's
    dequantise-then-matmul path evaluates it (one gather, one fp32 sum,
    reference ``src/runtime.py:379-414``).
    """
    groups, entries, d = (int(v) for v in codebooks.shape)
    if route.shape != code.shape:
        raise ValueError("route and code must have the same [rows, blocks] shape")
    ids = route.to(torch.int32) * entries + code.to(torch.int32)
    flat = codebooks.reshape(groups * entries, d)
    id_dtype = torch.uint8 if groups * entries <= 256 else torch.int16
    return make_plain_encoding([ids.to(id_dtype)], [flat], row_scale, in_features=in_features, block_size=d)
