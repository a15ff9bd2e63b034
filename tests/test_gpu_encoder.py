"""GPU encoder against the reference's own encoder (``tests/golden/encoder.npz``).

``wal_rvq_assign`` must return the reference's nearest entry for every block
except near-ties (equal distance up to fp32 rounding); ``fit_kmeans`` starts
from the reference's initial entries (same seeded draws) and must end at its
codebook up to fp32 rounding; ``encode_block_rvq`` must give the reference's
row and block scales bit for bit, nearly all of its stage ids, and an
encoding of the same quality that decodes through this package's kernels.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from tests import goldens
from tests.test_encoder import near_tie_ok
from wal2026_b200.block_vq import single_group
from wal2026_b200.encoder import assign_to_codebook, encode_block_rvq, fit_kmeans
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_assignment_matches_reference():
    fx = goldens.load("encoder")
    ids, dist = assign_to_codebook(torch.from_numpy(fx["blocks"]).to(DEV), torch.from_numpy(fx["fit_codebook"]).to(DEV))
    ids, dist = ids.cpu().numpy(), dist.cpu().numpy()
    assert near_tie_ok(fx["blocks"], fx["fit_codebook"], ids, fx["ids"]) <= 4
    same = ids == fx["ids"]
    assert np.allclose(dist[same], fx["min_dist"][same], rtol=1e-5, atol=1e-6)


def test_kmeans_fit_matches_reference():
    fx = goldens.load("encoder")
    sample = torch.from_numpy(fx["blocks"][: int(fx["sample_rows"])]).to(DEV)
    cb = fit_kmeans(sample, int(fx["fit_entries"]), int(fx["fit_iters"])).cpu().numpy()
    want = fx["fit_codebook"]
    assert np.abs(cb - want).max() <= 1e-5 * np.abs(want).max()


@pytest.mark.parametrize("tag,kw", [("plain", {}), ("split", dict(product_splits=2, stages_per_split=(2, 1),
                                                                     normalize_blocks="amax"))])
def test_encoder_matches_reference_encoder(tag, kw):
    fx = goldens.load("encoder")
    w = torch.from_numpy(fx["weight"]).to(DEV)
    enc = encode_block_rvq(w, block_size=8, codebook_size=64, num_stages=2, kmeans_iters=3, **kw)
    assert np.array_equal(enc.row_scale.cpu().numpy().view(np.uint16), fx[f"{tag}_rho"].view(np.uint16))
    if f"{tag}_block_scale" in fx:
        assert np.array_equal(enc.block_scale.cpu().numpy().view(np.uint16), fx[f"{tag}_block_scale"].view(np.uint16))
    for si, ids in enumerate(enc.stage_ids):
        agree = float((ids.cpu().numpy() == fx[f"{tag}_ids{si}"]).mean())
        assert agree >= 0.99, (si, agree)
        books = enc.codebooks[si].float().cpu().numpy()
        want = fx[f"{tag}_book{si}"].astype(np.float32)
        assert np.abs(books - want).max() <= 2e-3 * np.abs(want).max() + 1e-6
    assert abs(enc.sample_rel_mse - float(fx[f"{tag}_rel_mse"])) <= 0.02 * float(fx[f"{tag}_rel_mse"])
    # the encoding decodes through the packed kernels like any reference encoding
    mod = PackedGroupedBlockRVQLinear(single_group(enc)).to(DEV)
    x = torch.randn(3, 256, device=DEV).to(torch.bfloat16)
    y = torch.empty(3, 96, device=DEV, dtype=torch.float32)
    mod.gemv_into(x, y)
    groups = orc.groups_from_encoding(single_group(enc))
    if mod.has_corrections:  # block-normalised encodings carry block scales
        w_ref = orc.f32_to_bf16_bits(orc.reconstruct_typed(groups, 256, "bf16"))
    else:
        w_ref = orc.reconstruct_bits(groups, 256)
    ref = orc.linear_exact(x.cpu().view(torch.int16).numpy().view(np.uint16), w_ref)
    assert np.abs(y.cpu().numpy() - ref).max() <= 2e-3 * np.abs(ref).max()
