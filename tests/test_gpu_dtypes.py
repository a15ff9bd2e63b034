"""fp16 / fp32 activations, the fast numerics mode and dropped stages on the GPU.

Weights materialised by the library must equal the reference-made fixture
bits (``tests/golden/dtype_*.npz``, ``stage_drop_*.npz``) in every dtype and
both reconstruction modes; forward outputs are checked against the exact
product of those weights (fp32 result within 2e-3 of ||y||_inf, observed at
fp32 accumulation-order noise; 16-bit outputs within one ulp of that type).
Every call goes through the C ABI.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from tests import goldens
from tests.test_stage_drop import fixture_active, stage_drop_encoding
from wal2026_b200 import synthetic
from wal2026_b200.block_vq import single_group
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear, set_global_effective_stages

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 2e-3
DTYPE_CASES = ["dtype_r2_d8", "dtype_scaled_grouped", "dtype_route", "dtype_scaled_r1"]


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def assert_close(y: np.ndarray, ref: np.ndarray, tol: float = TOL) -> float:
    scale = float(np.abs(ref).max())
    err = float(np.abs(y.astype(np.float64) - ref.astype(np.float64)).max())
    assert err <= tol * scale, f"max err {err} > {tol} * {scale}"
    return err / max(scale, 1e-30)


def assert_within_ulp(y: np.ndarray, ref: np.ndarray, mant_bits: int) -> None:
    """16-bit outputs: one ulp of the output type plus fp32 accumulation noise near zero."""
    y, ref = y.astype(np.float64), ref.astype(np.float64)
    tol = np.abs(ref) * 2.0 ** -mant_bits + 1e-5 * np.abs(ref).max()
    assert np.all(np.abs(y - ref) <= tol), float(np.abs(y - ref).max())


def module(fx, strategy="per_group"):
    enc = goldens.encoding_from_fixture(fx)
    bias = goldens.bf16_tensor(fx["bias_bits"]) if "bias_bits" in fx else None
    return PackedGroupedBlockRVQLinear(enc, bias, matmul_strategy=strategy).to(DEV)


@pytest.mark.parametrize("name", DTYPE_CASES)
def test_reconstruct_weight_in_every_dtype_matches_reference(name):
    fx = goldens.load(name)
    mod = module(fx)
    assert np.array_equal(bits16(mod.reconstruct_weight(torch.float16)), fx["w16_bits"])
    w32 = mod.reconstruct_weight(torch.float32).cpu().numpy()
    assert np.array_equal(w32.view(np.uint32), fx["w32"].view(np.uint32))
    fast = module(fx, "full_weight_fast")
    assert np.array_equal(bits16(fast.reconstruct_weight_fast(torch.float16)), fx["wfast16_bits"])
    assert np.array_equal(bits16(fast.reconstruct_weight_fast(torch.bfloat16)), fx["wfast_bf16_bits"])
    wf32 = fast.reconstruct_weight_fast(torch.float32).cpu().numpy()
    assert np.array_equal(wf32.view(np.uint32), fx["wfast32"].view(np.uint32))


@pytest.mark.parametrize("name", DTYPE_CASES)
def test_forward_in_fp16_and_fp32_matches_reference(name):
    fx = goldens.load(name)
    mod = module(fx)
    for M, xb in goldens.x_inputs(fx).items():
        x16 = xb.to(torch.float16).to(DEV)
        y16 = mod(x16)
        assert y16.dtype == torch.float16
        ref16 = fx[f"y{M}_f16_ref32"]
        assert_within_ulp(y16.float().cpu().numpy(), ref16, 10)
        # the fp32 pre-rounding result through the typed GEMV
        y = torch.empty(M, mod.out_features, device=DEV, dtype=torch.float32)
        mod.gemv_into(x16, y)
        assert_close(y.cpu().numpy(), ref16)
        y32 = mod(xb.to(torch.float32).to(DEV))
        assert y32.dtype == torch.float32
        assert_close(y32.cpu().numpy(), fx[f"y{M}_f32_ref64"], tol=1e-5)


@pytest.mark.parametrize("name", DTYPE_CASES)
def test_fast_strategy_forward_matches_reference_fast_path(name):
    fx = goldens.load(name)
    mod = module(fx, "full_weight_fast")
    for M, xb in goldens.x_inputs(fx).items():
        y = torch.empty(M, mod.out_features, device=DEV, dtype=torch.float32)
        mod.gemv_into(xb.to(DEV), y)
        assert_close(y.cpu().numpy(), fx[f"y{M}_fast_ref32"])
        yb = mod(xb.to(DEV))
        assert_within_ulp(yb.float().cpu().numpy(), fx[f"y{M}_fast_ref32"], 7)


@pytest.mark.parametrize("name", ["stage_drop_r3", "stage_drop_r3_k1", "stage_drop_splits"])
def test_dropped_stages_match_reference_fast_path(name):
    fx = goldens.load(name)
    mod = PackedGroupedBlockRVQLinear(stage_drop_encoding(fx), matmul_strategy="full_weight_fast").to(DEV)
    full_bits = bits16(mod.reconstruct_weight())
    assert np.array_equal(full_bits, fx["w_bits"])  # reconstruct_weight ignores the stage setting
    set_global_effective_stages(mod, int(fx["k"]))
    assert mod._active_stages() == fixture_active(fx)
    assert np.array_equal(bits16(mod.reconstruct_weight_fast()), fx["w_fast_bits"])
    for M, xb in goldens.x_inputs(fx).items():
        y = torch.empty(M, mod.out_features, device=DEV, dtype=torch.float32)
        mod.gemv_into(xb.to(DEV), y)
        assert_close(y.cpu().numpy(), fx[f"y{M}_fast32"])
    # per_group sums every stage whatever the setting, as the reference does
    mod.matmul_strategy = "per_group"
    x = goldens.x_inputs(fx)
    M, xb = next(iter(x.items()))
    y = torch.empty(M, mod.out_features, device=DEV, dtype=torch.float32)
    mod.gemv_into(xb.to(DEV), y)
    ref = orc.linear_exact(bits16(xb), full_bits)
    assert_close(y.cpu().numpy(), ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("strategy,R", [("per_group", 2), ("full_weight_fast", 2), ("full_weight_fast", 1),
                                        ("per_group", 1)])
def test_prefill_gemm_in_fp16_and_fast_mode_matches_oracle(dtype, strategy, R):
    M, N, K = 300, 384, 520
    enc = single_group(synthetic.rvq_encoding(N, K, d=8, R=R, seed=M + R))
    mod = PackedGroupedBlockRVQLinear(enc, matmul_strategy=strategy).to(DEV)
    x = synthetic.activations(M, K, seed=7).to(dtype)
    y = torch.empty(M, N, device=DEV, dtype=torch.float32)
    status = torch.zeros(1, device=DEV, dtype=torch.int32)
    assert mod.gemm_into(x.to(DEV), y, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    wt = "f16" if dtype == torch.float16 else "bf16"
    mode = "fast" if strategy == "full_weight_fast" else "exact"
    w = orc.reconstruct_typed(orc.groups_from_encoding(enc), K, wt, mode).astype(np.float64)
    ref = x.float().numpy().astype(np.float64) @ w.T
    assert_close(y.cpu().numpy(), ref)
    yo = mod(x.to(DEV))  # large M: the same GEMM, output in x.dtype
    assert yo.dtype == dtype
    assert_within_ulp(yo.float().cpu().numpy(), ref, 10 if dtype == torch.float16 else 7)


@pytest.mark.parametrize("M", [1, 5, 17])
def test_fp16_gemv_every_slab_and_fast_mode(M):
    # token counts across the n-tile variants and slabs, fp16, both modes
    enc = single_group(synthetic.rvq_encoding(200, 512, d=8, R=2, seed=51))
    for strategy, mode in (("per_group", "exact"), ("per_group_fast", "fast")):
        mod = PackedGroupedBlockRVQLinear(enc, matmul_strategy=strategy).to(DEV)
        x = synthetic.activations(M, 512, seed=M).to(torch.float16)
        y = torch.empty(M, 200, device=DEV, dtype=torch.float32)
        mod.gemv_into(x.to(DEV), y)
        w = orc.reconstruct_typed(orc.groups_from_encoding(enc), 512, "f16", mode).astype(np.float64)
        assert_close(y.cpu().numpy(), x.float().numpy().astype(np.float64) @ w.T)
