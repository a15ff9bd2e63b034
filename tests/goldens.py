"""Helpers to load the reference-generated golden fixtures under ``tests/golden/``."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
SMALL_CASES = ["small_r2_d8", "small_r1_ragged", "small_r3_d16", "small_grouped", "small_route",
               "small_d32", "small_r4_wide"]


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
        groups.append({"stage_ids": ids, "codebooks": books, "row_scale": fx[f"g{gi}_rho"]})
        gi += 1
    return groups


def bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
