"""Llama stack construction and tensor-parallel shard shapes (CPU only, no forward)."""
from __future__ import annotations

import pytest
import torch

from wal2026_b200.llama import LLAMA_8B, LlamaShape, TPContext, dense_llama, rvq_llama
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear

TINY = LlamaShape(layers=2, hidden=512, mlp=1024, heads=8, kv_heads=4, vocab=1024)


def test_rvq_stack_builds_packed_projections():
    st = rvq_llama(TINY, device="cpu", seed=0)
    lin = [m for m in st.modules() if isinstance(m, PackedGroupedBlockRVQLinear)]
    assert len(lin) == 4 * TINY.layers
    qkv = st.layers[0].qkv
    hd = TINY.head_dim
    assert qkv.row_slices == ((0, 8 * hd), (8 * hd, 12 * hd), (12 * hd, 16 * hd))
    assert qkv.num_groups == 3 and qkv.codebooks.shape == (3, 2, 256, 8)
    assert st.layers[0].gate_up.out_features == 2 * TINY.mlp and st.layers[0].down.in_features == TINY.mlp
    # 2 bits per weight for the ids (d = 8, 2 stages of 1-byte ids)
    ids = sum(m.packed_ids.numel() for m in lin)
    weights = TINY.layers * (TINY.hidden * 16 * hd + TINY.hidden * 8 * hd + 2 * TINY.mlp * TINY.hidden
                             + TINY.hidden * TINY.mlp)
    assert ids * 4 == weights


@pytest.mark.parametrize("tp", [2, 4])
def test_tensor_parallel_shards(tp):
    for rank in range(tp):
        st = rvq_llama(TINY, device="cpu", seed=0, tp=TPContext(rank, tp))
        layer = st.layers[0]
        hd = TINY.head_dim
        assert layer.qkv.out_features == (TINY.heads + 2 * TINY.kv_heads) * hd // tp
        assert layer.o.in_features == TINY.heads * hd // tp and layer.o.out_features == TINY.hidden
        assert layer.down.in_features == TINY.mlp // tp
        assert st.lm_head.shape == (TINY.vocab // tp, TINY.hidden)


def test_tp_rejects_indivisible_heads():
    with pytest.raises(ValueError, match="divisible"):
        rvq_llama(TINY, device="cpu", tp=TPContext(0, 3))


def test_dense_twin_has_same_shapes():
    a = rvq_llama(TINY, device="cpu", seed=0)
    b = dense_llama(TINY, device="cpu", seed=0)
    for la, lb in zip(a.layers, b.layers):
        for name in ("qkv", "o", "gate_up", "down"):
            assert getattr(la, name).out_features == getattr(lb, name).out_features
            assert getattr(la, name).in_features == getattr(lb, name).in_features
    assert 4 * a.linear_bytes() < b.linear_bytes() < 8 * a.linear_bytes()  # codebooks weigh more on tiny layers


def test_8b_shape_constants():
    assert LLAMA_8B.head_dim == 128 and LLAMA_8B.hidden // 8 % 8 == 0
