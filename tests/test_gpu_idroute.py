"""ID-route GEMV and weight materialisation on the GPU, through the C ABI.

Weights bit-exact against the reference-made fixtures (fp16 reconstruct_weight
and its bf16 cast); GEMV fp32 output within 2e-3 of ||y||_inf of the reference
(fp32-accumulate oracle), bf16 output within one bf16 ulp; every token-count
variant and ragged K.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from wal2026_b200 import synthetic
from wal2026_b200.idroute import PackedIDRouteLinear

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def module_from_fixture(fx) -> PackedIDRouteLinear:
    ids = torch.from_numpy(fx["ids"].astype(np.int32))
    book = torch.from_numpy(fx["codebook_w_bits"].view(np.int16)).view(torch.float16)
    rho = torch.from_numpy(fx["rho_bits"].view(np.int16)).view(torch.float16).reshape(-1, 1)
    bias = None
    if "bias_f16_bits" in fx:
        bias = torch.from_numpy(fx["bias_f16_bits"].view(np.int16)).view(torch.float16)
    return PackedIDRouteLinear(ids, book, rho, bias).cuda()


def assert_close(y: np.ndarray, ref: np.ndarray, tol: float = 2e-3) -> None:
    err = float(np.max(np.abs(y - ref)))
    scale = float(np.max(np.abs(ref)))
    assert err <= tol * scale, f"max err {err} > {tol} * {scale}"


@pytest.mark.parametrize("name", ["idroute_small", "idroute_medium"])
def test_weights_and_outputs_match_reference_fixtures(name):
    fx = dict(np.load(GOLDEN / f"{name}.npz"))
    mod = module_from_fixture(fx)
    w16 = mod.reconstruct_weight(torch.float16)
    assert np.array_equal(bits(w16), fx["w16_bits"])
    wb = mod.reconstruct_weight(torch.bfloat16)
    assert np.array_equal(bits(wb), bits(w16.to(torch.bfloat16)))
    for key in fx:
        if key.startswith("x") and key.endswith("_bits"):
            M = key[1:-5]
            x = torch.from_numpy(fx[key].view(np.int16)).view(torch.bfloat16).cuda()
            y = torch.empty(x.shape[0], mod.out_features, device="cuda", dtype=torch.float32)
            mod.gemv_into(x, y)
            assert_close(y.cpu().numpy(), fx[f"y{M}_ref32"])
            yb = mod(x).float().cpu().numpy()
            assert_close(yb, fx[f"y{M}_ref32"], tol=8e-3)


@pytest.mark.parametrize("N,K,routes,M", [(1000, 520, 1536, 1), (512, 4096, 1536, 4), (300, 1032, 4000, 9),
                                          (64, 256, 32767, 16), (96, 136, 300, 17), (4096, 1024, 1536, 33)])
def test_random_shapes_against_oracle(N, K, routes, M):
    inp = synthetic.idroute_inputs(N, K, routes=routes, seed=N + M)
    mod = PackedIDRouteLinear(inp.ids, inp.codebook_w, inp.row_scale).cuda()
    cs = bits(mod.codebook_sum)
    rho = bits(inp.row_scale.reshape(-1))
    w = orc.idroute_weight_bits(inp.ids.numpy(), cs, rho)
    assert np.array_equal(bits(mod.reconstruct_weight(torch.bfloat16)), w)
    x = synthetic.activations(M, K, seed=M)
    ref = orc.linear_exact(bits(x), w)
    y = torch.empty(M, N, device="cuda", dtype=torch.float32)
    mod.gemv_into(x.cuda(), y)
    assert_close(y.cpu().numpy(), ref)


def test_strided_activation_rows():
    inp = synthetic.idroute_inputs(256, 512, routes=1000, seed=5)
    mod = PackedIDRouteLinear(inp.ids, inp.codebook_w, inp.row_scale).cuda()
    big = synthetic.activations(3, 520, seed=5).cuda()
    x = big[:, :512]  # row stride 520
    y = torch.empty(3, 256, device="cuda", dtype=torch.float32)
    mod.gemv_into(x, y)
    w = orc.idroute_weight_bits(inp.ids.numpy(), bits(mod.codebook_sum), bits(inp.row_scale.reshape(-1)))
    assert_close(y.cpu().numpy(), orc.linear_exact(bits(x.contiguous()), w))
