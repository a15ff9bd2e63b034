"""The CPU oracle reproduces the reference's own outputs (golden fixtures made by running it)."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from tests import goldens
from wal2026_b200 import synthetic
from wal2026_b200.block_vq import single_group


@pytest.mark.parametrize("name", goldens.SMALL_CASES)
def test_oracle_weight_bit_exact(name):
    fx = goldens.load(name)
    groups = goldens.groups_from_fixture(fx)
    w = orc.reconstruct_bits(groups, int(fx["K"]))
    assert np.array_equal(w, fx["w_bits"])
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(fx["w_sha256"])


@pytest.mark.parametrize("name", goldens.SMALL_CASES)
def test_oracle_forward_matches_reference(name):
    fx = goldens.load(name)
    groups = goldens.groups_from_fixture(fx)
    bias = fx.get("bias_bits")
    for key in fx:
        if not (key.startswith("x") and key.endswith("_bits")):
            continue
        M = int(key[1:-5])
        y = orc.forward_f32(fx[key], groups, int(fx["K"]), bias)
        ref32 = fx[f"y{M}_ref32"]
        tol = 2e-3 * np.abs(ref32).max()
        assert np.abs(y - ref32).max() <= 1e-5 * np.abs(ref32).max() <= tol
        # the reference's own bf16 output differs from rounding the oracle's fp32 value by <= 1 ulp
        y_bf = orc.bf16_bits_to_f32(orc.f32_to_bf16_bits(y))
        ref_bf = orc.bf16_bits_to_f32(fx[f"y{M}_ref_bf16"])
        ulp = np.maximum(np.abs(ref_bf), 1e-30) * 2.0 ** -7
        assert np.all(np.abs(y_bf - ref_bf) <= ulp)


def test_synthetic_inputs_match_fixture_digests():
    """The seeded generator still yields the exact bytes the fixtures were made from."""
    fx = goldens.load("small_r2_d8")
    enc = synthetic.rvq_encoding(37, 64, d=8, R=2, seed=11)
    for s, (ids, book) in enumerate(zip(enc.stage_ids, enc.codebooks)):
        assert goldens.sha(ids) == str(fx[f"g0_ids{s}_sha256"])
        assert goldens.sha(book) == str(fx[f"g0_book{s}_sha256"])
    assert goldens.sha(synthetic.activations(3, 64, seed=11)) == str(fx["x3_sha256"])


def test_oracle_full_cfg0_pinned():
    """Full-size config 0: oracle weight digest and outputs equal the reference's."""
    fx = goldens.load("cfg0")
    enc = synthetic.cfg0_encoding(0)
    g = enc.groups[0]
    for s, (ids, book) in enumerate(zip(g.stage_ids, g.codebooks)):
        assert goldens.sha(ids) == str(fx[f"g0_ids{s}_sha256"])
        assert goldens.sha(book) == str(fx[f"g0_book{s}_sha256"])
    assert goldens.sha(g.row_scale) == str(fx["g0_rho_sha256"])
    groups = orc.groups_from_encoding(enc)
    w = orc.reconstruct_bits(groups, 2048)
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(fx["w_sha256"])
    for M in (1, 4, 16):
        x = synthetic.activations(M, 2048, seed=0)
        assert goldens.sha(x) == str(fx[f"x{M}_sha256"])
        xb = x.view(torch.int16).numpy().view(np.uint16)
        y = orc.linear_exact(xb, w).astype(np.float32)
        ref32 = fx[f"y{M}_ref32"]
        assert np.abs(y - ref32).max() <= 1e-5 * np.abs(ref32).max()


def test_oracle_full_cfg1_pinned():
    """Full-size config 1 (route-codebook 4096 -> 14336): weight digest equals the reference's."""
    fx = goldens.load("cfg1")
    inp = synthetic.cfg1_inputs(1)
    enc = single_group(inp.encoding())
    g = enc.groups[0]
    assert goldens.sha(g.stage_ids[0]) == str(fx["g0_ids0_sha256"])
    assert goldens.sha(g.codebooks[0]) == str(fx["g0_book0_sha256"])
    groups = orc.groups_from_encoding(enc)
    w = orc.reconstruct_bits(groups, 4096)
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(fx["w_sha256"])
    x = synthetic.activations(1, 4096, seed=1)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    y = orc.linear_exact(xb, w[:2048]).astype(np.float32)
    ref32 = fx["y1_ref32"]
    assert np.abs(y - ref32).max() <= 1e-5 * np.abs(ref32).max()
    route, code = orc.unpack_route_code(g.stage_ids[0].numpy())
    assert np.array_equal(route, inp.route.numpy()) and np.array_equal(code, inp.code.numpy())


@pytest.mark.parametrize("name", [c for c in goldens.SMALL_CASES if "scaled" not in c])
def test_c_oracle_matches_reference(name):
    """The C restatement (CPU baseline) covers unscaled stages; scaled ones are the numpy oracle's."""
    from oracle import c_oracle

    fx = goldens.load(name)
    groups = goldens.groups_from_fixture(fx)
    K = int(fx["K"])
    assert np.array_equal(c_oracle.reconstruct(groups, K), fx["w_bits"])
    bias = fx.get("bias_bits")
    for M, x in goldens.x_inputs(fx).items():
        xb = x.view(torch.int16).numpy().view(np.uint16)
        y = c_oracle.forward(xb, groups, K, bias)
        ref = fx[f"y{M}_ref32"]
        assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()


def test_c_oracle_full_cfg0_weight_digest():
    from oracle import c_oracle

    fx = goldens.load("cfg0")
    w = c_oracle.reconstruct(orc.groups_from_encoding(synthetic.cfg0_encoding(0)), 2048)
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(fx["w_sha256"])
