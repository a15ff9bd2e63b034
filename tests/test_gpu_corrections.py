"""Per-block corrections on the GPU against the reference's own weights and outputs.

Encodings made by the reference's encoder (``tests/golden/corr_*``): the
corrected weight of ``wal_rvq_dequant_corrected`` in bf16 / fp16 / fp32 against
the reference's ``reconstruct_weight`` (the correction matrix products sum in
another order than the reference's CPU product, so a small share of rounded
weights may differ by one unit in the last place), and the fused corrected
GEMV (bf16, fp16, fp32 activations) and the large-M path against the exact
product of the reference's weights within the output tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from tests import goldens
from tests.test_corrections import CASES, assert_weights_match, bf16_ulp, f16_ulp, load_case

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-3


def bits16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def module(name):
    from wal2026_b200.runtime import PackedGroupedBlockRVQLinear

    fx, enc = load_case(name)
    bias = goldens.bf16_tensor(fx["bias_bits"]) if "bias_bits" in fx else None
    return fx, enc, PackedGroupedBlockRVQLinear(enc, bias).to(DEV)


def assert_close(y, ref, tol=TOL):
    ref = np.asarray(ref, dtype=np.float64)
    err = float(np.abs(np.asarray(y, dtype=np.float64) - ref).max())
    assert err <= tol * float(np.abs(ref).max()), (err, float(np.abs(ref).max()))


@pytest.mark.parametrize("name", CASES)
def test_corrected_weights_match_reference(name):
    fx, enc, mod = module(name)
    wb = orc.bf16_bits_to_f32(bits16(mod.reconstruct_weight(torch.bfloat16)))
    assert_weights_match(wb, orc.bf16_bits_to_f32(fx["w_bits"]), bf16_ulp)
    w16 = mod.reconstruct_weight(torch.float16).float().cpu().numpy()
    assert_weights_match(w16, fx["w16_bits"].view(np.float16).astype(np.float32), f16_ulp)
    w32 = mod.reconstruct_weight(torch.float32).cpu().numpy().astype(np.float64)
    want = fx["w32"].astype(np.float64)
    assert np.abs(w32 - want).max() <= 1e-6 * np.abs(want).max()
    # the fast strategies fall back to the full reconstruction, as in the reference
    mod.matmul_strategy = "full_weight_fast"
    assert torch.equal(mod.reconstruct_weight_fast(), mod.reconstruct_weight())


@pytest.mark.parametrize("name", CASES)
def test_corrected_forward_matches_reference(name):
    fx, enc, mod = module(name)
    w_ref = fx["w_bits"]
    for M, xb in goldens.x_inputs(fx).items():
        ref = fx[f"y{M}_ref32"]
        y = torch.empty(M, mod.out_features, device=DEV, dtype=torch.float32)
        mod.gemv_into(xb.to(DEV), y)
        assert_close(y.cpu().numpy(), ref)
        yb = mod(xb.to(DEV))
        assert yb.dtype == torch.bfloat16
        assert_close(yb.float().cpu().numpy(), ref, tol=8e-3)
        # fp16 and fp32 activations: against the product of the reference's weights of that dtype
        for dt, wkey in ((torch.float16, "w16_bits"), (torch.float32, "w32")):
            w = fx[wkey].view(np.float16).astype(np.float64) if dt == torch.float16 else fx[wkey].astype(np.float64)
            x = xb.to(dt)
            r = x.double().numpy() @ w.T
            if "bias_bits" in fx:
                r = r + orc.bf16_bits_to_f32(fx["bias_bits"]).astype(np.float64)[None, :]
            yt = mod(x.to(DEV))
            assert yt.dtype == dt
            assert_close(yt.float().cpu().numpy(), r, tol=8e-3 if dt == torch.float16 else 1e-5)
    # many tokens: the corrected weight once, then a library GEMM
    x = torch.randn(100, mod.in_features).to(torch.bfloat16)
    r = x.double().numpy() @ orc.bf16_bits_to_f32(w_ref).astype(np.float64).T
    if "bias_bits" in fx:
        r = r + orc.bf16_bits_to_f32(fx["bias_bits"]).astype(np.float64)[None, :]
    assert_close(mod(x.to(DEV)).float().cpu().numpy(), r, tol=8e-3)
