"""Encoding maps: load and save the reference's on-disk map of pre-encoded layers.

The file format is the reference's (``src/encoding_io.py:10-94``): a
``torch.save`` payload ``{"version": 1, "encodings": {name: grouped}}`` where
every grouped encoding is ``{"groups": [...], "row_slices": [...],
"original_shape": [...]}`` and every group is a dict of the
``BlockRVQEncoding`` fields (tensors on the CPU).  Maps written by the
reference load here unchanged and vice versa (the keys must match for that);
the loader uses ``torch.load(weights_only=True)``, which accepts exactly the
tensors, lists, dicts, strings and numbers the format contains.

``load_grouped_encoding_map`` + ``runtime.replace_with_preencoded_packed_block_rvq``
is the reference's serving flow for pre-encoded models.
"""
from __future__ import annotations

from pathlib import Path
from typing import Optional

import torch

from .block_vq import BlockRVQEncoding, GroupedBlockRVQEncoding

FORMAT_VERSION = 1


def _serialize_block(enc: BlockRVQEncoding) -> dict:
    def cpu(t):
        return None if t is None else t.detach().cpu()

    return {
        "stage_ids": [cpu(t) for t in enc.stage_ids],
        "codebooks": [cpu(t) for t in enc.codebooks],
        "stage_value_dims": [int(v) for v in enc.stage_value_dims],
        "stages_per_split": [int(v) for v in enc.stages_per_split],
        "stage_scales": cpu(enc.stage_scales),
        "residual_correction": str(enc.residual_correction),
        "residual_signs": cpu(enc.residual_signs),
        "residual_scale": cpu(enc.residual_scale),
        "row_scale": cpu(enc.row_scale),
        "block_scale": cpu(enc.block_scale),
        "transform_kind": str(enc.transform_kind),
        "transform_matrix": cpu(enc.transform_matrix),
        "transform_bias": cpu(enc.transform_bias),
        "product_splits": int(enc.product_splits),
        "original_shape": [int(v) for v in enc.original_shape],
        "padded_cols": int(enc.padded_cols),
        "block_size": int(enc.block_size),
        "sample_rel_mse": float(enc.sample_rel_mse),
    }


def _deserialize_block(d: dict, device: Optional[torch.device]) -> BlockRVQEncoding:
    def mv(t):
        return t if (t is None or device is None) else t.to(device)

    return BlockRVQEncoding(
        stage_ids=tuple(mv(t) for t in d["stage_ids"]),
        codebooks=tuple(mv(t) for t in d["codebooks"]),
        stage_value_dims=tuple(int(v) for v in d["stage_value_dims"]),
        stages_per_split=tuple(int(v) for v in d["stages_per_split"]),
        stage_scales=mv(d["stage_scales"]),
        residual_correction=str(d["residual_correction"]),
        residual_signs=mv(d["residual_signs"]),
        residual_scale=mv(d["residual_scale"]),
        row_scale=mv(d["row_scale"]),
        block_scale=mv(d["block_scale"]),
        transform_kind=str(d["transform_kind"]),
        transform_matrix=mv(d["transform_matrix"]),
        transform_bias=mv(d["transform_bias"]),
        product_splits=int(d["product_splits"]),
        original_shape=tuple(int(v) for v in d["original_shape"]),
        padded_cols=int(d["padded_cols"]),
        block_size=int(d["block_size"]),
        sample_rel_mse=float(d["sample_rel_mse"]),
    )


def serialize_grouped_encoding(enc: GroupedBlockRVQEncoding) -> dict:
    return {"groups": [_serialize_block(g) for g in enc.groups],
            "row_slices": [[int(a), int(b)] for a, b in enc.row_slices],
            "original_shape": [int(v) for v in enc.original_shape]}


def deserialize_grouped_encoding(d: dict, device: Optional[torch.device] = None) -> GroupedBlockRVQEncoding:
    return GroupedBlockRVQEncoding(
        groups=tuple(_deserialize_block(g, device) for g in d["groups"]),
        row_slices=tuple(tuple(int(v) for v in s) for s in d["row_slices"]),
        original_shape=tuple(int(v) for v in d["original_shape"]),
    )


def save_grouped_encoding_map(path: str | Path, encodings: dict[str, GroupedBlockRVQEncoding]) -> Path:
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    torch.save({"version": FORMAT_VERSION,
                "encodings": {name: serialize_grouped_encoding(e) for name, e in encodings.items()}}, target)
    return target


def load_grouped_encoding_map(path: str | Path,
                              device: Optional[torch.device] = None) -> dict[str, GroupedBlockRVQEncoding]:
    payload = torch.load(Path(path), map_location="cpu", weights_only=True)
    if int(payload.get("version", 0)) != FORMAT_VERSION:
        raise ValueError(f"unsupported encoding map version: {payload.get('version')}")
    return {name: deserialize_grouped_encoding(d, device) for name, d in payload["encodings"].items()}
