"""ID-route linear on the CPU: the oracle against the reference's own outputs,
the module's route table against the reference's, and the packed id layout."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from wal2026_b200 import synthetic
from wal2026_b200.idroute import PackedIDRouteLinear, pack_ids

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["idroute_small", "idroute_medium"]


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


@pytest.mark.parametrize("name", CASES)
def test_oracle_weight_matches_reference_bit_for_bit(name):
    fx = load(name)
    w16 = orc.idroute_weight_f16_bits(fx["ids"], fx["codebook_sum_bits"], fx["rho_bits"])
    assert np.array_equal(w16, fx["w16_bits"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_forward_matches_reference(name):
    fx = load(name)
    w = orc.idroute_weight_bits(fx["ids"], fx["codebook_sum_bits"], fx["rho_bits"])
    bias = None
    if "bias_f16_bits" in fx:
        bias = orc.f32_to_bf16_bits(fx["bias_f16_bits"].view(np.float16).astype(np.float32))
    for key in fx:
        if key.startswith("x") and key.endswith("_bits"):
            M = key[1:-5]
            y = orc.linear_exact(fx[key], w, bias)
            ref = fx[f"y{M}_ref32"]
            assert np.max(np.abs(y - ref)) <= 1e-6 * max(np.max(np.abs(ref)), 1e-30)
            # the reference's bf16 output is one rounding of the same sum (up to fp32 order)
            yb = fx[f"y{M}_ref_bf16"].view(np.uint16)
            ours = orc.f32_to_bf16_bits(y.astype(np.float32))
            assert np.mean(ours != yb) < 0.02


@pytest.mark.parametrize("name", CASES)
def test_module_route_table_matches_reference(name):
    fx = load(name)
    ids = torch.from_numpy(fx["ids"].astype(np.int32))
    book = torch.from_numpy(fx["codebook_w_bits"].view(np.int16)).view(torch.float16)
    rho = torch.from_numpy(fx["rho_bits"].view(np.int16)).view(torch.float16).reshape(-1, 1)
    mod = PackedIDRouteLinear(ids, book, rho)
    assert np.array_equal(mod.codebook_sum.view(torch.int16).numpy().view(np.uint16), fx["codebook_sum_bits"])


def unpack(packed: np.ndarray, N: int, K: int) -> np.ndarray:
    """Independent reader of the layout documented for wal_idroute_pack."""
    chunks = -(-K // 128)
    out = np.zeros((N, K), dtype=np.int16)
    b = packed.view(np.uint8)
    for n in range(N):
        t, rr = divmod(n, 16)
        h, r = divmod(rr, 8)
        for k in range(K):
            c, cc = divmod(k, 128)
            g, in32 = divmod(cc, 32)
            u, rest = divmod(in32, 16)
            q, j = divmod(rest, 4)
            off = (t * chunks + c) * 4096 + (h * 4 + g) * 512 + (r * 4 + q) * 16 + u * 8 + j * 2
            out[n, k] = b[off:off + 2].view(np.int16)[0]
    return out


@pytest.mark.parametrize("N,K", [(40, 136), (17, 256), (33, 8)])
def test_packed_layout_round_trips(N, K):
    inp = synthetic.idroute_inputs(N, K, routes=700, seed=N + K)
    packed = pack_ids(inp.ids, 700).numpy()
    assert np.array_equal(unpack(packed, N, K), inp.ids.numpy().astype(np.int16))


def test_validation():
    inp = synthetic.idroute_inputs(16, 64, routes=10, seed=1)
    with pytest.raises(ValueError, match="range"):
        PackedIDRouteLinear(inp.ids + 10, inp.codebook_w, inp.row_scale)
    with pytest.raises(ValueError, match="multiple of 8"):
        PackedIDRouteLinear(inp.ids[:, :60], inp.codebook_w, inp.row_scale)
    mod = PackedIDRouteLinear(inp.ids, inp.codebook_w, inp.row_scale)
    with pytest.raises(ValueError, match="CUDA"):
        mod(torch.zeros(1, 64, dtype=torch.bfloat16))
