"""The allocation-free decode attention entry point against the workspace one.

wal_decode_attention_static serves callers that cannot call cudaMalloc (an
engine plugin given no workspace, a serving loop that must not stall on the
synchronisation an allocation brings): its scratch is an array compiled into
the library.  Through the C ABI it must give the same bits as
wal_decode_attention on consecutive calls whose shapes change (so each call
finds the array as the previous one left it), and refuse shapes beyond the
array.  The file sorts last so a run that stops at the first failure has run
every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import pytest
import torch

from wal2026_b200 import _abi
from wal2026_b200.decode_ops import decode_attention, decode_attention_workspace

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(B, hq, hkv, hd, L, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B, hq * hd, device=DEV, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, hkv, L, hd, device=DEV, generator=g).to(torch.bfloat16)
    return q, kc, vc


def _static(q, kc, vc, n, out):
    B, hkv, L, hd = (int(v) for v in kc.shape)
    hq = int(q.shape[1]) // hd
    return _abi.load().wal_decode_attention_static(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), B, hq,
                                                   hkv, hd, L, n, float(hd) ** -0.5, out.data_ptr(), out.stride(0),
                                                   _abi.stream_handle(q.device))


def test_static_scratch_matches_workspace_entry_on_consecutive_calls():
    # shapes change between calls, so each call's partials overlay what the previous one left
    for B, hq, hkv, hd, L, n, seed in ((8, 32, 8, 128, 2048, 2001, 1), (3, 8, 2, 64, 600, 517, 2),
                                      (8, 32, 8, 128, 2048, 2048, 3)):
        q, kc, vc = _inputs(B, hq, hkv, hd, L, seed)
        want = torch.empty(B, hq * hd, device=DEV, dtype=torch.bfloat16)
        decode_attention(q, kc, vc, n, want, decode_attention_workspace(B, hq, hkv, hd, L, DEV))
        for _ in range(2):  # two calls in a row: the counters came back to zero
            got = torch.full_like(want, float("nan"))
            assert _static(q, kc, vc, n, got) == _abi.WAL_OK
            torch.cuda.synchronize()
            assert torch.equal(got, want)


def test_static_scratch_rejects_shapes_beyond_its_size():
    # 33 * 128 = 4224 (batch, kv head) counters: more than the 4096 the array holds
    q, kc, vc = _inputs(33, 128, 128, 64, 8, 4)
    out = torch.empty(33, 128 * 64, device=DEV, dtype=torch.bfloat16)
    assert _static(q, kc, vc, 8, out) == _abi.WAL_ERR_BUFFER_TOO_SMALL
    # 128 sequences x 8 kv heads x 1 split x 8 heads x 128 fp32 partials = 4 MiB, above 4 MiB - 16 KiB
    q, kc, vc = _inputs(128, 64, 8, 128, 64, 5)
    out = torch.empty(128, 64 * 128, device=DEV, dtype=torch.bfloat16)
    assert _static(q, kc, vc, 64, out) == _abi.WAL_ERR_BUFFER_TOO_SMALL
    # the same cache read at 4 sequences fits and still matches
    want = torch.empty(4, 64 * 128, device=DEV, dtype=torch.bfloat16)
    decode_attention(q[:4], kc[:4], vc[:4], 64, want, decode_attention_workspace(4, 64, 8, 128, 64, DEV))
    got = torch.empty_like(want)
    assert _static(q[:4], kc[:4], vc[:4], 64, got) == _abi.WAL_OK
    torch.cuda.synchronize()
    assert torch.equal(got, want)
