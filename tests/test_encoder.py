"""Encoder: the oracle's nearest-entry assignment against the reference's (``tests/golden/encoder.npz``,
made by the reference's ``_assign_to_codebook`` / ``_fit_kmeans`` / ``encode_block_residual_vq``),
and the GPU encoder's argument checks.  Assignments may differ only where the two best entries are
within fp32 rounding of each other (the reference's CPU matrix product sums in its own order).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from tests import goldens


def near_tie_ok(blocks, codebook, got, want, rel=1e-5):
    """Indices that differ must be near-ties: equal distance up to fp32 rounding."""
    x = blocks.astype(np.float64)
    c = codebook.astype(np.float64)
    d = ((x[:, None, :] - c[None, :, :]) ** 2).sum(-1)
    bad = np.nonzero(got != want)[0]
    for i in bad:
        a, b = d[i, got[i]], d[i, want[i]]
        assert abs(a - b) <= rel * max(abs(a), abs(b), 1e-12), (i, a, b)
    return len(bad)


def test_oracle_assignment_matches_reference():
    fx = goldens.load("encoder")
    ids, dist = orc.assign_to_codebook(fx["blocks"], fx["fit_codebook"])
    assert near_tie_ok(fx["blocks"], fx["fit_codebook"], ids, fx["ids"]) <= 4
    same = ids == fx["ids"]
    assert np.allclose(dist[same], fx["min_dist"][same], rtol=1e-5, atol=1e-6)


def test_gpu_encoder_rejects_unsupported_options():
    from wal2026_b200.encoder import encode_block_rvq

    w = torch.zeros(4, 16)
    with pytest.raises(ValueError, match="CUDA"):
        encode_block_rvq(w)
    if torch.cuda.is_available():
        with pytest.raises(ValueError, match="plain stages"):
            encode_block_rvq(w.cuda(), transform_kind="dct")
