"""Helpers to load the reference-generated golden fixtures under ``tests/golden/``."""
from __future__ import annotations

import dataclasses
import hashlib
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
SMALL_CASES = ["small_r2_d8", "small_r1_ragged", "small_r3_d16", "small_grouped", "small_route",
               "small_d32", "small_r4_wide", "small_scaled_r2", "small_scaled_r1", "small_scaled_grouped",
               "small_product_splits"]


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def sha(t) -> str:
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        t = t.numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


def groups_from_fixture(fx: dict) -> list[dict]:
    groups = []
    gi = 0
    while f"g{gi}_rho" in fx:
        ids, books = [], []
        s = 0
        while f"g{gi}_ids{s}" in fx:
            ids.append(fx[f"g{gi}_ids{s}"])
            books.append(fx[f"g{gi}_book{s}"])
            s += 1
        groups.append({"stage_ids": ids, "codebooks": books, "row_scale": fx[f"g{gi}_rho"],
                       "stage_scales": fx.get(f"g{gi}_scales")})
        gi += 1
    return groups


def bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def encoding_from_fixture(fx: dict):
    """Rebuild the grouped encoding (torch tensors) a fixture was generated from."""
    from wal2026_b200.block_vq import GroupedBlockRVQEncoding, make_plain_encoding

    K = int(fx["K"])
    groups, slices, row0 = [], [], 0
    for g in groups_from_fixture(fx):
        d = int(g["codebooks"][0].shape[1])
        ids = [torch.from_numpy(np.ascontiguousarray(a)) for a in g["stage_ids"]]
        books = [torch.from_numpy(np.ascontiguousarray(b)) for b in g["codebooks"]]
        rho = torch.from_numpy(np.ascontiguousarray(g["row_scale"]))
        enc = make_plain_encoding(ids, books, rho, in_features=K, block_size=d)
        if g["stage_scales"] is not None:
            enc = dataclasses.replace(enc, stage_scales=torch.from_numpy(np.ascontiguousarray(g["stage_scales"])))
        if "product_splits" in fx:  # the reference encoder's split metadata (codebooks are full width)
            enc = dataclasses.replace(enc, product_splits=int(fx["product_splits"]),
                                      stages_per_split=tuple(int(v) for v in fx["stages_per_split"]),
                                      stage_value_dims=tuple(int(v) for v in fx["stage_value_dims"]))
        n = int(ids[0].shape[0])
        groups.append(enc)
        slices.append((row0, row0 + n))
        row0 += n
    return GroupedBlockRVQEncoding(groups=tuple(groups), row_slices=tuple(slices), original_shape=(row0, K))


def x_inputs(fx: dict) -> dict[int, torch.Tensor]:
    out = {}
    for key in fx:
        if key.startswith("x") and key.endswith("_bits"):
            out[int(key[1:-5])] = bf16_tensor(fx[key])
    return out
