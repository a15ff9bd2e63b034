"""Variable effective stages (reference src/runtime.py:352-377, :568-598, :2274-2327) on the CPU.

The fixtures ``tests/golden/stage_drop_*.npz`` were made by the reference
itself: ``set_global_effective_stages(module, k)`` under ``full_weight_fast``,
recording the active stage indices, the bf16 weight of
``reconstruct_weight_fast`` (bf16 accumulation of the active stages) and its
forward.  Checked here: the module API keeps the same active indices and
setter counts, the derived packed stream of the active stages equals packing
the stage-subset encoding bit for bit, and the oracle's exact active-stage
result stays within the output tolerance of the reference's fast path.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch
from torch import nn

from oracle import rvq_oracle as orc
from tests import goldens
from wal2026_b200.block_vq import GroupedBlockRVQEncoding
from wal2026_b200.packing import pack_grouped
from wal2026_b200.runtime import (PackedGroupedBlockRVQLinear, set_effective_stages_by_name,
                                  set_effective_stages_from_map, set_global_effective_stages)

CASES = ["stage_drop_r3", "stage_drop_r3_k1", "stage_drop_splits"]


def stage_drop_encoding(fx: dict) -> GroupedBlockRVQEncoding:
    enc = goldens.encoding_from_fixture(fx)
    sps = np.atleast_2d(fx["stages_per_split"])
    groups = tuple(dataclasses.replace(g, product_splits=len(row), stages_per_split=tuple(int(v) for v in row))
                   for g, row in zip(enc.groups, sps))
    return dataclasses.replace(enc, groups=groups)


def subset_encoding(enc: GroupedBlockRVQEncoding, active) -> GroupedBlockRVQEncoding:
    """The encoding restricted to the union of the active stages, zero codebooks where a group drops one."""
    union = sorted(set().union(*active))
    groups = []
    for g, act in zip(enc.groups, active):
        books = tuple(g.codebooks[s] if s in act else torch.zeros_like(g.codebooks[s]) for s in union)
        groups.append(dataclasses.replace(g, stage_ids=tuple(g.stage_ids[s] for s in union), codebooks=books,
                                          stage_value_dims=tuple(g.block_size for _ in union),
                                          stages_per_split=(len(union),), product_splits=1))
    return dataclasses.replace(enc, groups=tuple(groups))


def fixture_active(fx: dict) -> tuple[tuple[int, ...], ...]:
    out, gi = [], 0
    while f"g{gi}_active" in fx:
        out.append(tuple(int(v) for v in fx[f"g{gi}_active"]))
        gi += 1
    return tuple(out)


@pytest.mark.parametrize("name", CASES)
def test_active_stage_indices_match_reference(name):
    fx = goldens.load(name)
    mod = PackedGroupedBlockRVQLinear(stage_drop_encoding(fx), matmul_strategy="full_weight_fast")
    assert set_global_effective_stages(mod, int(fx["k"])) == int(fx["groups_updated"])
    assert tuple(g._compute_active_stage_indices() for g in mod.groups) == fixture_active(fx)
    assert mod._active_stages() == fixture_active(fx)
    # the default strategy sums every stage whatever the setting, as in the reference
    mod.matmul_strategy = "per_group"
    assert mod._active_stages() is None


@pytest.mark.parametrize("name", CASES)
def test_stage_view_equals_packing_the_stage_subset(name):
    fx = goldens.load(name)
    enc = stage_drop_encoding(fx)
    mod = PackedGroupedBlockRVQLinear(enc, matmul_strategy="per_group_fast")
    set_global_effective_stages(mod, int(fx["k"]))
    R, packed, books, scales = mod._stage_view(mod._active_stages())
    want = pack_grouped(subset_encoding(enc, fixture_active(fx)))
    assert R == int(want.geometry.num_stages) < mod.num_stages
    assert torch.equal(packed, want.packed_ids) and torch.equal(books, want.codebooks)
    assert scales is None
    assert packed.numel() * mod.num_stages == mod.packed_ids.numel() * R  # only the active stages' bytes


@pytest.mark.parametrize("name", CASES)
def test_oracle_fast_result_matches_reference_fast_forward(name):
    fx = goldens.load(name)
    groups = goldens.groups_from_fixture(fx)
    K = int(fx["K"])
    sub = []
    for g, act in zip(groups, fixture_active(fx)):
        sub.append({"stage_ids": [g["stage_ids"][s] for s in act], "codebooks": [g["codebooks"][s] for s in act],
                    "row_scale": g["row_scale"], "stage_scales": None})
    w = orc.f32_to_bf16_bits(orc.reconstruct_typed(sub, K, "bf16", "fast"))
    assert np.array_equal(w, fx["w_fast_bits"])
    for M, x in goldens.x_inputs(fx).items():
        y = orc.linear_exact(x.view(torch.int16).numpy().view(np.uint16), w)
        ref = fx[f"y{M}_fast32"]
        assert float(np.abs(y - ref).max()) <= 1e-5 * float(np.abs(ref).max())


def test_module_level_setters_count_like_the_reference():
    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = nn.Module()
            self.mlp = nn.Module()
            fx = goldens.load("stage_drop_r3_k1")
            self.self_attn.q_proj = PackedGroupedBlockRVQLinear(stage_drop_encoding(fx),
                                                                matmul_strategy="full_weight_fast")
            self.mlp.up_proj = PackedGroupedBlockRVQLinear(stage_drop_encoding(fx), matmul_strategy="full_weight_fast")

    model = nn.Module()
    model.layers = nn.ModuleList([Block(), Block()])
    assert set_global_effective_stages(model, 2) == 8  # two groups per linear
    assert set_effective_stages_by_name(model, 1, None) == {"attn": 2, "mlp": 0, "other": 0}
    assert model.layers[0].self_attn.q_proj._active_stages() == ((0,), (0,))
    assert model.layers[0].mlp.up_proj._active_stages() == ((0, 1), (0, 1))
    assert set_effective_stages_from_map(model, {"layers.1.mlp.up_proj": 1, "nope": 2}) == 1
    assert model.layers[1].mlp.up_proj._active_stages() == ((0,), (0,))
    assert set_global_effective_stages(model, 3) == 8
    assert model.layers[1].mlp.up_proj._active_stages() is None  # every stage active again
