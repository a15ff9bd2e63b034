"""Encoding maps: the reference's on-disk format loads here, round-trips, packs and
drives the pre-encoded model surgery (CPU only: construction, no forward)."""
from __future__ import annotations

import dataclasses
from pathlib import Path

import pytest
import torch
from torch import nn

from tests import goldens
from wal2026_b200 import synthetic
from wal2026_b200.block_vq import single_group
from wal2026_b200.encoding_io import load_grouped_encoding_map, save_grouped_encoding_map
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear, replace_with_preencoded_packed_block_rvq

MAP = goldens.GOLDEN / "encoding_map_small.pt"


def expected():
    """The encodings the fixture map was written from (same seeds and scales)."""
    a = single_group(synthetic.rvq_encoding(48, 136, d=8, R=2, seed=18))
    a = dataclasses.replace(a, groups=(dataclasses.replace(a.groups[0],
                                                           stage_scales=torch.tensor([0.8125, 1.3125],
                                                                                     dtype=torch.float16)),))
    b = synthetic.grouped_encoding([16, 24, 9], 128, d=8, R=2, seed=14)
    return {"model.layers.0.mlp.up_proj": a, "model.layers.0.self_attn.q_proj": b}


def same(e1, e2) -> None:
    assert e1.row_slices == e2.row_slices and tuple(e1.original_shape) == tuple(e2.original_shape)
    for g1, g2 in zip(e1.groups, e2.groups):
        for f in dataclasses.fields(g1):
            v1, v2 = getattr(g1, f.name), getattr(g2, f.name)
            if isinstance(v1, tuple) and v1 and isinstance(v1[0], torch.Tensor):
                assert all(torch.equal(a, b) for a, b in zip(v1, v2)), f.name
            elif isinstance(v1, torch.Tensor):
                assert torch.equal(v1, v2), f.name
            else:
                assert v1 == v2 or (tuple(v1) == tuple(v2) if isinstance(v1, (list, tuple)) else False), f.name


def test_reference_written_map_loads_unchanged():
    maps = load_grouped_encoding_map(MAP)
    exp = expected()
    assert set(maps) == set(exp)
    for name in exp:
        same(maps[name], exp[name])


def test_round_trip(tmp_path: Path):
    maps = load_grouped_encoding_map(MAP)
    path = save_grouped_encoding_map(tmp_path / "m.pt", maps)
    again = load_grouped_encoding_map(path)
    for name in maps:
        same(maps[name], again[name])


def test_rejects_unknown_version(tmp_path: Path):
    torch.save({"version": 2, "encodings": {}}, tmp_path / "v2.pt")
    with pytest.raises(ValueError, match="version"):
        load_grouped_encoding_map(tmp_path / "v2.pt")


def test_loaded_map_packs_and_drives_the_surgery():
    maps = load_grouped_encoding_map(MAP)
    model = nn.Module()
    model.model = nn.Module()
    model.model.layers = nn.ModuleList([nn.Module()])
    layer = model.model.layers[0]
    layer.mlp = nn.Module()
    layer.self_attn = nn.Module()
    layer.mlp.up_proj = nn.Linear(136, 48, bias=False)
    layer.self_attn.q_proj = nn.Linear(128, 49, bias=True)
    stats = replace_with_preencoded_packed_block_rvq(model, maps)
    assert {s["name"] for s in stats} == set(maps)
    up = model.model.layers[0].mlp.up_proj
    assert isinstance(up, PackedGroupedBlockRVQLinear)
    assert up.stage_scales is not None and torch.equal(up.stage_scales, torch.tensor([[0.8125, 1.3125]]))
    q = model.model.layers[0].self_attn.q_proj
    assert isinstance(q, PackedGroupedBlockRVQLinear) and q.num_groups == 3 and q.bias is not None
