"""Per-block corrections (reference src/runtime.py:389-412) on the CPU: encodings made by the reference's
own encoder (block scale, sign residual, DCT / Hadamard / randomised Hadamard / PCA / polar transforms),
loaded through this package's encoding-map reader, packed with their side arrays and reconstructed by
the oracle restatement against the reference's weights.

The reference multiplies the correction matrices with a CPU matrix product
whose summation order is its own; the oracle rounds the exact dot products
once.  Weights may therefore differ in the last bit before the rounding to
the weight type: the share of weights that differ after rounding is bounded
here (observed: zero or a handful per fixture) and no weight may differ by
more than one unit in the last place of its type.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import rvq_oracle as orc
from tests import goldens
from wal2026_b200 import _abi
from wal2026_b200.encoding_io import load_grouped_encoding_map
from wal2026_b200.packing import pack_corrections
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear

CASES = ["corr_sign_amax", "corr_dct_l2", "corr_hadamard_d16", "corr_grouped_pca_rand", "corr_polar"]
MAX_DIFF_SHARE = 2e-3  # weights whose rounded value may differ (last-bit order effects)


def load_case(name):
    fx = goldens.load(name)
    enc = load_grouped_encoding_map(goldens.GOLDEN / f"{name}.pt")["layer"]
    return fx, enc


def assert_weights_match(got: np.ndarray, want: np.ndarray, ulp_of) -> None:
    diff = got != want
    assert diff.mean() <= MAX_DIFF_SHARE, diff.mean()
    if diff.any():
        g, w = got[diff].astype(np.float64), want[diff].astype(np.float64)
        assert np.all(np.abs(g - w) <= ulp_of(np.abs(w)) * 1.0000001)


def bf16_ulp(a):
    return 2.0 ** (np.floor(np.log2(np.maximum(a, 1e-30))) - 7)


def f16_ulp(a):
    return 2.0 ** (np.floor(np.log2(np.maximum(a, 6.1e-5))) - 10)


@pytest.mark.parametrize("name", CASES)
def test_oracle_reconstructs_reference_weights_with_corrections(name):
    fx, enc = load_case(name)
    groups = orc.groups_from_encoding(enc)
    K = int(fx["K"])
    wb = orc.bf16_bits_to_f32(orc.f32_to_bf16_bits(orc.reconstruct_typed(groups, K, "bf16")))
    assert_weights_match(wb, orc.bf16_bits_to_f32(fx["w_bits"]), bf16_ulp)
    w16 = orc.reconstruct_typed(groups, K, "f16")
    assert_weights_match(w16, fx["w16_bits"].view(np.float16).astype(np.float32), f16_ulp)
    # fp32 weights carry the matrix-product order effects unrounded (observed <= 2e-7 of the largest weight)
    w32 = orc.reconstruct_typed(groups, K, "f32").astype(np.float64)
    want = fx["w32"].astype(np.float64)
    assert np.abs(w32 - want).max() <= 1e-6 * np.abs(want).max()


@pytest.mark.parametrize("name", CASES)
def test_correction_side_arrays(name):
    fx, enc = load_case(name)
    corr = pack_corrections(enc)
    assert corr is not None
    for gi, g in enumerate(enc.groups):
        f = int(corr.group_flags[gi])
        assert bool(f & _abi.WAL_CORR_SIGN) == bool(fx["signs"][gi])
        assert bool(f & _abi.WAL_CORR_BLOCK_SCALE) == bool(fx["block_scale"][gi])
        kind = str(fx["kinds"][gi])
        assert bool(f & _abi.WAL_CORR_POLAR) == (kind == "polar")
        assert bool(f & _abi.WAL_CORR_MATRIX) == (kind not in ("none", "polar"))
        assert bool(f & _abi.WAL_CORR_BIAS) == (g.transform_bias is not None)
    mod = PackedGroupedBlockRVQLinear(enc)
    assert mod.has_corrections and mod.sum_mode() == _abi.WAL_SUM_EXACT
    fast = PackedGroupedBlockRVQLinear(enc, matmul_strategy="full_weight_fast")
    assert fast.sum_mode() == _abi.WAL_SUM_EXACT and fast._active_stages() is None  # the reference falls back too


def test_sign_matrix_and_transforms_are_the_references():
    from wal2026_b200.packing import dct_matrix, hadamard_matrix, rand_hadamard_matrix

    for n in (8, 16, 32):
        assert np.array_equal(rand_hadamard_matrix(n).numpy(), orc._rand_hadamard(n))
        assert np.array_equal(hadamard_matrix(n).numpy(), orc._fixed_transform("hadamard", n))
        assert np.array_equal(dct_matrix(n).numpy(), orc._fixed_transform("dct", n))
