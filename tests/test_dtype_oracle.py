"""The oracle's fp16 / fp32 and fast-mode reconstructions against reference-made fixtures.

``tests/golden/dtype_*.npz`` hold, from the reference itself, the per_group
weights ``reconstruct_weight(torch.float16 / torch.float32)``, the fast
reconstruction ``reconstruct_weight_fast`` in bf16 / fp16 / fp32 and the
forward outputs in fp16 and fp32; ``stage_drop_*.npz`` the fast weights with
dropped stages.  The oracle must reproduce every weight bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import rvq_oracle as orc
from tests import goldens

DTYPE_CASES = ["dtype_r2_d8", "dtype_scaled_grouped", "dtype_route", "dtype_scaled_r1"]


@pytest.mark.parametrize("name", DTYPE_CASES)
def test_oracle_exact_weights_in_every_dtype(name):
    fx = goldens.load(name)
    groups, K = goldens.groups_from_fixture(fx), int(fx["K"])
    w16 = orc.reconstruct_typed(groups, K, "f16", "exact")
    assert np.array_equal(w16.astype(np.float16).view(np.uint16), fx["w16_bits"])
    w32 = orc.reconstruct_typed(groups, K, "f32", "exact")
    assert np.array_equal(w32.view(np.uint32), fx["w32"].view(np.uint32))
    # the bf16 form is the one the other fixtures pin
    wb = orc.reconstruct_typed(groups, K, "bf16", "exact")
    assert np.array_equal(orc.f32_to_bf16_bits(wb), orc.reconstruct_bits(groups, K))


@pytest.mark.parametrize("name", DTYPE_CASES)
def test_oracle_fast_weights_in_every_dtype(name):
    fx = goldens.load(name)
    groups, K = goldens.groups_from_fixture(fx), int(fx["K"])
    wf16 = orc.reconstruct_typed(groups, K, "f16", "fast")
    assert np.array_equal(wf16.astype(np.float16).view(np.uint16), fx["wfast16_bits"])
    wfb = orc.reconstruct_typed(groups, K, "bf16", "fast")
    assert np.array_equal(orc.f32_to_bf16_bits(wfb), fx["wfast_bf16_bits"])
    wf32 = orc.reconstruct_typed(groups, K, "f32", "fast")
    assert np.array_equal(wf32.view(np.uint32), fx["wfast32"].view(np.uint32))


@pytest.mark.parametrize("name", ["stage_drop_r3", "stage_drop_r3_k1", "stage_drop_splits"])
def test_oracle_fast_weights_with_dropped_stages(name):
    fx = goldens.load(name)
    groups, K = goldens.groups_from_fixture(fx), int(fx["K"])
    sub, gi = [], 0
    for g in groups:
        act = [int(v) for v in fx[f"g{gi}_active"]]
        sub.append({"stage_ids": [g["stage_ids"][s] for s in act], "codebooks": [g["codebooks"][s] for s in act],
                    "row_scale": g["row_scale"], "stage_scales": None})
        gi += 1
    w = orc.reconstruct_typed(sub, K, "bf16", "fast")
    assert np.array_equal(orc.f32_to_bf16_bits(w), fx["w_fast_bits"])


@pytest.mark.parametrize("name", DTYPE_CASES)
def test_reference_outputs_are_the_products_of_these_weights(name):
    # sanity of the fixtures: the reference's fp16 / fp32 forward outputs sit
    # within the output tolerance of the exact product of its own weights
    fx = goldens.load(name)
    for key in fx:
        if not (key.startswith("x") and key.endswith("_bits")):
            continue
        M = int(key[1:-5])
        ref32 = fx[f"y{M}_f16_ref32"].astype(np.float64)
        y16 = fx[f"y{M}_f16_bits"].view(np.float16).astype(np.float64)
        assert np.abs(y16 - ref32).max() <= 4e-3 * np.abs(ref32).max()
        r64 = fx[f"y{M}_f32_ref64"]
        assert np.abs(fx[f"y{M}_f32"].astype(np.float64) - r64).max() <= 1e-5 * np.abs(r64).max()
