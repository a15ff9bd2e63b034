"""Tensor-parallel sharding on the CPU.

* ``shard_packed`` (cutting a packed module's buffers) equals packing
  ``shard_encoding`` (cutting the encoding), buffer for buffer;
* the sharded forward, summed (row-parallel) or gathered (column-parallel)
  across world-size-2 ``gloo`` ranks, equals the single-rank oracle forward.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import rvq_oracle as orc
from wal2026_b200 import synthetic
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear
from wal2026_b200.tp import COLUMN, ROW, shard_bounds, shard_encoding, shard_packed

CASES = {
    "qkv_like_d8_r2": ([256, 128, 128], 512, 8, 2),
    "one_group_d16_r1": ([512], 1024, 16, 1),
    "two_groups_d8_r3": ([256, 256], 1024, 8, 3),
}


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("mode", [COLUMN, ROW])
@pytest.mark.parametrize("size", [2, 4])
def test_packed_shard_equals_packed_encoding_shard(case, mode, size):
    rows, K, d, R = CASES[case]
    enc = synthetic.grouped_encoding(rows, K, d=d, R=R, seed=3)
    full = PackedGroupedBlockRVQLinear(enc)
    for rank in range(size):
        a = shard_packed(full, rank, size, mode)
        b = PackedGroupedBlockRVQLinear(shard_encoding(enc, rank, size, mode))
        assert (a.in_features, a.out_features, a.row_slices) == (b.in_features, b.out_features, b.row_slices)
        for name in ("packed_ids", "tile_table", "codebooks", "row_scale"):
            assert torch.equal(getattr(a, name), getattr(b, name)), (name, rank)


def test_shard_bounds_rejects_ragged_splits():
    with pytest.raises(ValueError, match="whole"):
        shard_bounds(1000, 0, 4, 16, "rows")
    assert shard_bounds(1024, 3, 4, 128, "in_features") == (768, 1024)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, size: int, port: int, mode: str, case: str, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        rows, K, d, R = CASES[case]
        enc = synthetic.grouped_encoding(rows, K, d=d, R=R, seed=3)
        x = synthetic.activations(3, K, seed=5)
        xb = x.view(torch.int16).numpy().view(np.uint16)
        shard = shard_encoding(enc, rank, size, mode)
        k_local = int(shard.original_shape[1])
        groups = orc.groups_from_encoding(shard)
        w = orc.reconstruct_bits(groups, k_local)
        if mode == ROW:
            k0, k1 = shard_bounds(K, rank, size, 16 * d, "in_features")
            y = torch.from_numpy(orc.linear_exact(np.ascontiguousarray(xb[:, k0:k1]), w))
            dist.all_reduce(y)  # the exchange step: sum of partials
        else:
            y_local = torch.from_numpy(orc.linear_exact(xb, w))
            parts = [torch.empty_like(y_local) for _ in range(size)]
            dist.all_gather(parts, y_local)
            # rank-major gather -> group-major rows: each group's slices in rank order
            cols, off = [], [0] * size
            for n in rows:
                step = n // size
                for r in range(size):
                    cols.append(parts[r][:, off[r]:off[r] + step])
                    off[r] += step
            y = torch.cat(cols, dim=1)
        if rank == 0:
            ref = orc.linear_exact(xb, orc.reconstruct_bits(orc.groups_from_encoding(enc), K))
            out.put(float(np.max(np.abs(y.numpy() - ref)) / max(np.max(np.abs(ref)), 1e-30)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", [COLUMN, ROW])
def test_sharded_forward_over_gloo_matches_single_rank_oracle(mode):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, mode, "qkv_like_d8_r2", out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    rel = out.get(timeout=5)
    # float64 accumulations summed in another order: equal to rounding
    assert rel < 1e-12, rel
