"""Tensor-parallel exchange emulated on one GPU, checked against the CPU oracle.

A row-parallel linear (o_proj / down_proj) is split along its input blocks
into P shards.  Each emulated rank r has its own exchange region on cuda:0;
``wal_rvq_gemv_push`` of shard r stores its tagged fp32 partial into every
region's receive slot for sender r, and ``wal_tp_reduce_rmsnorm`` on region r
sums the P partials in rank order, adds the residual and applies the RMSNorm.
The launches go on one stream in the order push, push, ..., reduce, reduce,
so every reduction starts after all pushes have finished: its bounded wait
finds every word already fresh and never depends on a kernel running
beside it.

The reduced output (residual 0, so h = bf16(sum of partials)) is compared
with the oracle's unsharded fp32 forward (the reference's dequantise-then-
matmul, ``src/runtime.py:379-414`` and ``:1501-1507``): within one bf16 ulp
plus fp32 accumulation-order noise, and identical on every emulated rank.
The RMSNorm output is compared with the same normalisation of the oracle
result.  This is the multi-rank data path of the decode step, run on the
one GPU the driver's test box has.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import rvq_oracle as orc
from wal2026_b200 import _abi, synthetic
from wal2026_b200.block_vq import single_group
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear
from wal2026_b200.tp import ROW, shard_packed

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
SLOTS = 4


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


class _Regions:
    """P exchange regions on one device with the layout of ``tp.PeerExchange``."""

    def __init__(self, P: int, max_rows: int, width: int):
        self.P, self.width = P, width
        self.slot_elems = max_rows * width
        nbytes = 4096 + SLOTS * P * self.slot_elems * 8
        self.buf = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(P)]
        self.base = [b.data_ptr() for b in self.buf]
        self.status = torch.zeros(1, dtype=torch.int32, device=DEV)

    def recv_off(self, slot: int, src: int) -> int:
        return 4096 + ((slot * self.P + src) * self.slot_elems) * 8

    def push(self, slot: int, r: int) -> _abi.TPPush:
        p = _abi.TPPush()
        p.num_ranks, p.rank, p.ld_dst = self.P, r, self.width
        for q in range(self.P):
            p.dst[q] = self.base[q] + self.recv_off(slot, r)
        p.epoch = self.base[r] + slot * 128
        return p


def _row_parallel_step(shards, xs, reg: _Regions, slot: int, hs, norm_w, xouts) -> None:
    lib = _abi.load()
    stream = _abi.stream_handle(DEV)
    pushes = [reg.push(slot, r) for r in range(reg.P)]
    for r, (lin, x) in enumerate(zip(shards, xs)):
        _abi.check(lib.wal_rvq_gemv_push(ctypes.byref(lin.layer_struct()), x.data_ptr(), x.shape[0], x.stride(0),
                                         ctypes.byref(pushes[r]), stream), "wal_rvq_gemv_push")
    for r in range(reg.P):
        M, N = hs[r].shape
        _abi.check(lib.wal_tp_reduce_rmsnorm(reg.base[r] + reg.recv_off(slot, 0), reg.P, reg.slot_elems, reg.width,
                                             reg.base[r] + slot * 128, reg.base[r] + 1024 + slot * 128,
                                             hs[r].data_ptr(), hs[r].stride(0), norm_w.data_ptr(), 1e-5,
                                             xouts[r].data_ptr(), xouts[r].stride(0), M, N, reg.status.data_ptr(),
                                             stream), "wal_tp_reduce_rmsnorm")


@pytest.mark.parametrize("P", [2, 4, 8])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_emulated_row_parallel_exchange_matches_unsharded_oracle(P, M):
    N, K = 1024, 4096
    enc = single_group(synthetic.rvq_encoding(N, K, d=8, R=2, seed=40 + P))
    full = PackedGroupedBlockRVQLinear(enc).to(DEV)
    shards = [shard_packed(full, r, P, ROW) for r in range(P)]
    kp = K // P
    reg = _Regions(P, 16, N)
    norm_w = (1.0 + 0.1 * torch.randn(N, generator=torch.Generator().manual_seed(P))).to(torch.bfloat16).to(DEV)
    groups = orc.groups_from_encoding(enc)
    for call in range(SLOTS + 2):  # every slot, two of them twice: tags advance per call
        slot = call % SLOTS
        x = synthetic.activations(M, K, seed=100 * P + call)
        xs = [x[:, r * kp:(r + 1) * kp].contiguous().to(DEV) for r in range(P)]
        hs = [torch.zeros(M, N, dtype=torch.bfloat16, device=DEV) for _ in range(P)]
        xouts = [torch.empty(M, N, dtype=torch.bfloat16, device=DEV) for _ in range(P)]
        _row_parallel_step(shards, xs, reg, slot, hs, norm_w, xouts)
        torch.cuda.synchronize()
        assert int(reg.status.item()) == 0
        for r in range(1, P):  # rank-order sum: every rank holds the same bits
            assert torch.equal(hs[r], hs[0]) and torch.equal(xouts[r], xouts[0])
        ref = orc.forward_f32(_bits(x), groups, K).astype(np.float64)
        got = orc.bf16_bits_to_f32(_bits(hs[0])).astype(np.float64)
        tol = np.abs(ref) * 2.0 ** -8 + 1e-5 * np.abs(ref).max()  # rounding to bf16 + fp32 order noise
        assert np.all(np.abs(got - ref) <= tol), (call, float(np.abs(got - ref).max()))
        # RMSNorm of the reduced h against the same math in float64
        hn = got / np.sqrt((got ** 2).mean(axis=1, keepdims=True) + 1e-5)
        want = hn * orc.bf16_bits_to_f32(_bits(norm_w)).astype(np.float64)[None, :]
        xo = orc.bf16_bits_to_f32(_bits(xouts[0])).astype(np.float64)
        assert np.all(np.abs(xo - want) <= np.abs(want) * 2.0 ** -7 + 1e-6 * np.abs(want).max()), call
