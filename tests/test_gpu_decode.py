"""Decode glue kernels, the push exchange (one rank) and the fused decode step, on the GPU.

The glue kernels are checked against the PyTorch operators they replace in
``DecoderLayer.forward``; the push exchange (GEMV storing tagged words into a
receive slot, then the waiting reduction) against the plain GEMV followed by
the local reduction; the bounded wait by words whose tag never arrives.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from wal2026_b200 import _abi
from wal2026_b200.decode_ops import (decode_attention, decode_attention_workspace, residual_rmsnorm, rope_kv_append,
                                     silu_mul)
from wal2026_b200.llama import LlamaShape, _rope, dense_llama, rvq_llama
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear
from wal2026_b200.tp import PeerExchange

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def _bf16_close(a: torch.Tensor, b: torch.Tensor, ulps: float = 1.0) -> None:
    a, b = a.float(), b.float()
    tol = ulps * b.abs() * 2.0 ** -7 + 1e-6 * b.abs().max()
    bad = (a - b).abs() > tol
    assert not bool(bad.any()), f"{int(bad.sum())} elements differ; max {float((a - b).abs().max())}"


@pytest.mark.parametrize("M,N", [(1, 4096), (5, 2048), (16, 8192), (3, 16384)])
def test_residual_rmsnorm_matches_torch(M, N):
    g = _gen(M * 7 + N)
    h = torch.randn(M, N, device=DEV, generator=g).to(torch.bfloat16)
    part = torch.randn(M, N, device=DEV, generator=g) * 0.5
    w = (1.0 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(torch.bfloat16)
    h_ref = h + part.to(torch.bfloat16)
    x_ref = F.rms_norm(h_ref, (N,), w, 1e-5)
    x = torch.empty_like(h)
    residual_rmsnorm(h, w, 1e-5, x, partial=part)
    torch.cuda.synchronize()
    assert torch.equal(h, h_ref)  # the residual add rounds exactly like the bf16 torch add
    _bf16_close(x, x_ref)
    # norm only (no partial): h unchanged
    h2 = h.clone()
    residual_rmsnorm(h2, w, 1e-5, x)
    assert torch.equal(h2, h)
    _bf16_close(x, F.rms_norm(h, (N,), w, 1e-5))


@pytest.mark.parametrize("M,hq,hkv,hd", [(1, 32, 8, 128), (4, 4, 1, 128), (3, 8, 2, 64)])
def test_rope_kv_append_matches_torch(M, hq, hkv, hd):
    g = _gen(hq * 13 + M)
    L, pos = 40, 17
    qkv = torch.randn(M, (hq + 2 * hkv) * hd, device=DEV, generator=g).to(torch.bfloat16)
    inv = 1.0 / (500000.0 ** (torch.arange(0, hd, 2, device=DEV, dtype=torch.float32) / hd))
    ang = float(pos) * inv
    cos, sin = torch.cat((ang, ang)).cos(), torch.cat((ang, ang)).sin()
    kc = torch.randn(M, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(M, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    q, k, v = qkv.split([hq * hd, hkv * hd, hkv * hd], dim=-1)
    q_ref = _rope(q.view(M, hq, hd), cos, sin).reshape(M, hq * hd)
    kc_ref[:, :, pos] = _rope(k.view(M, hkv, hd), cos, sin)
    vc_ref[:, :, pos] = v.view(M, hkv, hd)
    q_out = torch.empty(M, hq * hd, device=DEV, dtype=torch.bfloat16)
    rope_kv_append(qkv, hq, hkv, hd, cos, sin, pos, q_out, kc, vc)
    torch.cuda.synchronize()
    assert torch.equal(q_out, q_ref)
    assert torch.equal(kc, kc_ref) and torch.equal(vc, vc_ref)


@pytest.mark.parametrize("M,I", [(1, 14336), (8, 3584), (32, 1000)])
def test_silu_mul_matches_torch(M, I):
    g = _gen(M + I)
    gu = (2.0 * torch.randn(M, 2 * I, device=DEV, generator=g)).to(torch.bfloat16)
    out = torch.empty(M, I, device=DEV, dtype=torch.bfloat16)
    silu_mul(gu, out)
    ref = F.silu(gu[:, :I]) * gu[:, I:]
    torch.cuda.synchronize()
    _bf16_close(out, ref)
    assert float((out.float() != ref.float()).float().mean()) < 1e-3


@pytest.mark.parametrize("B,hq,hkv,hd,L,n", [(1, 32, 8, 128, 2049, 2049), (3, 8, 2, 64, 600, 517), (2, 4, 4, 128, 40, 1),
                                           (1, 64, 8, 128, 4096, 4000), (5, 8, 1, 128, 300, 300),
                                           (64, 8, 1, 128, 4097, 4097)])
def test_decode_attention_matches_reference_math(B, hq, hkv, hd, L, n):
    g = _gen(B * 100 + n)
    q = torch.randn(B, hq * hd, device=DEV, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    out = torch.empty(B, hq * hd, device=DEV, dtype=torch.bfloat16)
    ws = decode_attention_workspace(B, hq, hkv, hd, L, DEV)
    decode_attention(q, kc, vc, n, out, ws)
    # float64 reference on the same bf16 inputs
    G = hq // hkv
    qd = q.double().view(B, hkv, G, hd)
    kd, vd = kc[:, :, :n].double(), vc[:, :, :n].double()
    s = torch.einsum("bhgd,bhtd->bhgt", qd, kd) / hd ** 0.5
    ref = torch.einsum("bhgt,bhtd->bhgd", torch.softmax(s, dim=-1), vd).reshape(B, hq * hd)
    err = float((out.double() - ref).abs().max())
    assert err <= 1e-2 * float(ref.abs().max()) + 1e-3, err
    again = torch.empty_like(out)
    decode_attention(q, kc, vc, n, again, ws)  # counters came back to zero: same bits
    assert torch.equal(out, again)


@pytest.mark.parametrize("B,hq,hkv,hd,L", [(1, 32, 8, 128, 1024), (2, 8, 2, 64, 700)])
def test_decode_attention_reuses_one_workspace_while_n_grows(B, hq, hkv, hd, L):
    # a decode loop sizes one workspace for its longest context and reuses it as
    # n grows; the split count is not monotone in n (for B = 1, hkv = 8 it drops
    # from 19 to 17 at n = 609), so each call must find its counters at zero
    g = _gen(B * 31 + L)
    q = torch.randn(B, hq * hd, device=DEV, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    ws = decode_attention_workspace(B, hq, hkv, hd, L, DEV)
    for n in list(range(600, 621)) + list(range(L - 8, L + 1)):
        got = torch.full((B, hq * hd), float("nan"), device=DEV, dtype=torch.bfloat16)
        decode_attention(q, kc, vc, n, got, ws)
        want = torch.empty_like(got)
        decode_attention(q, kc, vc, n, want, decode_attention_workspace(B, hq, hkv, hd, n, DEV))
        torch.cuda.synchronize()
        assert torch.equal(got, want), n


def _layer(N, K, seed=0):
    return PackedGroupedBlockRVQLinear.random([N], K, generator=_gen(seed), device=DEV)


@pytest.mark.parametrize("M", [1, 4, 20])
def test_push_exchange_one_rank_matches_local_reduction(M):
    N, K = 2048, 4096
    lin = _layer(N, K, seed=M)
    ex = PeerExchange(0, 1, 32, N, torch.device(DEV))
    try:
        g = _gen(100 + M)
        w = (1.0 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(torch.bfloat16)
        h0 = torch.randn(M, N, device=DEV, generator=g).to(torch.bfloat16)
        for call in range(6):  # every slot, some twice: epochs advance per call
            x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
            h_push, h_ref = h0.clone(), h0.clone()
            xo_push, xo_ref = torch.empty_like(h0), torch.empty_like(h0)
            slot = call % PeerExchange.SLOTS
            ex.push_gemv(lin, x, slot)
            ex.reduce_residual_norm(slot, h_push, w, 1e-5, xo_push)
            y32 = torch.empty(M, N, device=DEV, dtype=torch.float32)
            lin.gemv_into(x, y32)
            residual_rmsnorm(h_ref, w, 1e-5, xo_ref, partial=y32)
            torch.cuda.synchronize()
            assert torch.equal(h_push, h_ref) and torch.equal(xo_push, xo_ref), call
        ex.check_status()
    finally:
        ex.close()


def test_push_exchange_replays_in_a_cuda_graph():
    N, K, M = 1024, 2048, 2
    lin = _layer(N, K, seed=9)
    ex = PeerExchange(0, 1, M, N, torch.device(DEV))
    try:
        w = torch.ones(N, device=DEV, dtype=torch.bfloat16)
        x = torch.randn(M, K, device=DEV).to(torch.bfloat16)
        h = torch.zeros(M, N, device=DEV, dtype=torch.bfloat16)
        xo = torch.empty_like(h)
        ex.push_gemv(lin, x, 0)
        ex.reduce_residual_norm(0, h, w, 1e-5, xo)
        torch.cuda.synchronize()
        one = h.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for s in range(PeerExchange.SLOTS + 1):
                ex.push_gemv(lin, x, s % PeerExchange.SLOTS)
                ex.reduce_residual_norm(s % PeerExchange.SLOTS, h, w, 1e-5, xo)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        ex.check_status()
        # h accumulated 1 + 3 * 5 rounded additions of the same bf16 output
        ref = one.clone()
        for _ in range(3 * (PeerExchange.SLOTS + 1)):
            ref = ref + one
        assert torch.equal(h, ref)
        del graph
    finally:
        ex.close()


def test_peer_wait_times_out_with_a_status_instead_of_hanging():
    lib = _abi.load()
    M, N = 1, 1024
    recv = torch.zeros(2 * M * N, dtype=torch.int32, device=DEV)  # words whose tag never becomes 1
    counters = torch.zeros(64, dtype=torch.int32, device=DEV)     # epoch at [0], done at [32]
    h = torch.randn(M, N, device=DEV).to(torch.bfloat16)
    h_before = h.clone()
    x = torch.zeros_like(h)
    w = torch.ones(N, device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = lib.wal_tp_reduce_rmsnorm(recv.data_ptr(), 1, M * N, N, counters.data_ptr(), counters[32:].data_ptr(),
                                   h.data_ptr(), N, w.data_ptr(), 1e-5, x.data_ptr(), N, M, N, status.data_ptr(),
                                   _abi.stream_handle())
    assert st == 0
    torch.cuda.synchronize()  # returns after the ~2 s bounded wait
    assert int(status.item()) == _abi.WAL_ERR_PEER_TIMEOUT
    assert torch.equal(h, h_before) and not bool(x.any())
    assert int(counters[0].item()) == 0  # the call count did not advance
    # the context is still usable
    assert float(torch.ones(4, device=DEV).sum()) == 4.0


TINY = LlamaShape(layers=2, hidden=512, mlp=1024, heads=8, kv_heads=4, vocab=1024)


@pytest.mark.parametrize("ctor", [rvq_llama, dense_llama])
@pytest.mark.parametrize("batch", [1, 3])
def test_fused_decode_step_matches_operator_by_operator(ctor, batch):
    st = ctor(TINY, device=DEV, seed=1)
    st.allocate_cache(batch, 33, seed=2, consistent=True)
    tokens = torch.randint(0, TINY.vocab, (batch,), device=DEV, generator=_gen(3))
    cos, sin = st.rope_tables(32)
    ref = st.decode_step(tokens, 32, cos, sin).float()
    st.allocate_cache(batch, 33, seed=2, consistent=True)
    out = st.decode_step_fused(tokens, 32, cos, sin).float()
    torch.cuda.synchronize()
    err = float((out - ref).abs().max()) / float(ref.abs().max())
    assert err < 2e-2, err
