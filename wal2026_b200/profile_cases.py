"""Small workloads for profiling one kernel at a time: ``python -m wal2026_b200.profile_cases <case>``.

Each case builds its inputs on ``cuda:0`` (seeded), runs the kernel three times
and synchronises, so an ``ncu -k <kernel> -c <n>`` capture ends by itself in
seconds and holds a few hundred MB on the device at most.

  cfg1_gemv    config 1 route-codebook linear 4096 -> 14336 (d = 16, 16 Zipf
               routes x 256 codes), M = 1 GEMV (activations staged whole)
  gemv_window  Block-RVQ 16384 x 4096 (d = 8, R = 2), M = 16 GEMV: the
               activations do not fit beside the codebooks and stream through
               the CTA's window ring
  idroute_mlp  ID-route linear 4096 -> 14336 (1536 routes), M = 1 GEMV
  attention    decode attention, Llama-3-8B heads (32 q / 8 kv, head dim 128),
               batch 8 over 2048 cached positions
  prefill_gate_up  tcgen05 prefill GEMM, Llama-3-8B gate/up projection
               (2 x 14336 rows x 4096, d = 8, R = 2), 2048 tokens
  tp_breakdown per-kernel time of one Llama-3-8B decoder layer at the shard
               shapes of tensor parallelism 1/2/4/8, batch 1 and 32 (timed
               with CUDA events, not a profiler capture)
"""
from __future__ import annotations

import sys

import torch

from . import synthetic
from .decode_ops import decode_attention, decode_attention_workspace
from .idroute import PackedIDRouteLinear
from .runtime import PackedGroupedBlockRVQLinear, RouteCodebookLinear

DEV = torch.device("cuda:0")


def _gen(seed: int) -> torch.Generator:
    return torch.Generator(device=DEV).manual_seed(seed)


def cfg1_gemv() -> None:
    inp = synthetic.route_inputs(14336, 4096, d=16, G=16, seed=1)
    mod = RouteCodebookLinear.from_routes(inp.route, inp.code, inp.codebooks, inp.row_scale, in_features=4096).to(DEV)
    x = synthetic.activations(1, 4096, seed=1).to(DEV)
    y = torch.empty(1, 14336, device=DEV, dtype=torch.float32)
    for _ in range(3):
        mod.gemv_into(x, y)


def gemv_window() -> None:
    mod = PackedGroupedBlockRVQLinear.random([16384], 4096, generator=_gen(2), device=DEV)
    x = torch.randn(16, 4096, device=DEV, generator=_gen(3)).to(torch.bfloat16)
    y = torch.empty(16, 16384, device=DEV, dtype=torch.float32)
    for _ in range(3):
        mod.gemv_into(x, y)


def idroute_mlp() -> None:
    mod = PackedIDRouteLinear.random(14336, 4096, routes=1536, generator=_gen(5), device=DEV)
    x = torch.randn(1, 4096, device=DEV, generator=_gen(6)).to(torch.bfloat16)
    y = torch.empty(1, 14336, device=DEV, dtype=torch.bfloat16)
    for _ in range(3):
        mod.gemv_into(x, y)


def attention() -> None:
    B, hq, hkv, hd, n = 8, 32, 8, 128, 2048
    g = _gen(7)
    q = torch.randn(B, hq * hd, device=DEV, generator=g).to(torch.bfloat16)
    k = torch.randn(B, hkv, n, hd, device=DEV, generator=g).to(torch.bfloat16)
    v = torch.randn(B, hkv, n, hd, device=DEV, generator=g).to(torch.bfloat16)
    out = torch.empty(B, hq * hd, device=DEV, dtype=torch.bfloat16)
    ws = decode_attention_workspace(B, hq, hkv, hd, n, DEV)
    for _ in range(3):
        decode_attention(q, k, v, n, out, ws)


def prefill_gate_up() -> None:
    mod = PackedGroupedBlockRVQLinear.random([14336, 14336], 4096, generator=_gen(8), device=DEV)
    x = torch.randn(2048, 4096, device=DEV, generator=_gen(9)).to(torch.bfloat16)
    y = torch.empty(2048, 28672, device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(3):
        if not mod.gemm_into(x, y, status):
            raise RuntimeError("the prefill GEMM does not cover this layer")
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError("prefill GEMM reported a pipeline timeout")


def tp_breakdown(tp: int = 8, batch: int = 1, context: int = 2048) -> None:
    """Per-kernel device time of one Llama-3-8B decoder layer at tensor-parallel shard shapes, on one GPU.

    Each launch group of ``LlamaStack.decode_step_fused`` runs alone, 200
    times in one CUDA graph, timed with CUDA events; the exchange kernels push
    to ``tp`` receive regions in this GPU's memory (the NVLink stores and the
    wait for peers are not part of this figure).  Prints one JSON line.
    """
    import ctypes
    import json

    from . import _abi
    from .decode_ops import residual_rmsnorm, rope_kv_append, silu_mul
    from .llama import LLAMA_8B
    from .tp import COLUMN, ROW, shard_packed

    s = LLAMA_8B
    hd = s.head_dim
    hq, hkv, mlp = s.heads // tp, s.kv_heads // tp, s.mlp // tp
    g = _gen(11)

    def lin(rows, k, mode):
        full = PackedGroupedBlockRVQLinear.random(rows, k, generator=g, device=DEV)
        return full if tp == 1 else shard_packed(full, 0, tp, mode)

    qkv = lin([s.heads * hd, s.kv_heads * hd, s.kv_heads * hd], s.hidden, COLUMN)
    o = lin([s.hidden], s.heads * hd, ROW)
    gu = lin([s.mlp, s.mlp], s.hidden, COLUMN)
    down = lin([s.hidden], s.mlp, ROW)
    bf = torch.bfloat16
    x = torch.randn(batch, s.hidden, device=DEV, generator=g).to(bf)
    h = torch.randn(batch, s.hidden, device=DEV, generator=g).to(bf)
    nw = torch.ones(s.hidden, device=DEV, dtype=bf)
    yqkv = torch.empty(batch, qkv.out_features, device=DEV, dtype=bf)
    q = torch.empty(batch, hq * hd, device=DEV, dtype=bf)
    kc = torch.randn(batch, hkv, context + 1, hd, device=DEV, generator=g).to(bf)
    vc = torch.randn(batch, hkv, context + 1, hd, device=DEV, generator=g).to(bf)
    attn = torch.empty(batch, hq * hd, device=DEV, dtype=bf)
    ws = decode_attention_workspace(batch, hq, hkv, hd, context + 1, DEV)
    ygu = torch.empty(batch, 2 * mlp, device=DEV, dtype=bf)
    act = torch.empty(batch, mlp, device=DEV, dtype=bf)
    cos = torch.ones(hd, device=DEV)
    sin = torch.zeros(hd, device=DEV)
    xo = torch.empty_like(h)
    # tp receive regions on this GPU (layout of tp.PeerExchange, one slot)
    slot_elems = batch * s.hidden
    regions = [torch.zeros(4096 + tp * slot_elems * 8, dtype=torch.uint8, device=DEV) for _ in range(tp)]
    pushes = []
    for src in range(tp):  # emulated sender src stores into every region's src block
        push = _abi.TPPush()
        push.num_ranks, push.rank, push.ld_dst = tp, src, s.hidden
        for r in range(tp):
            push.dst[r] = regions[r].data_ptr() + 4096 + src * slot_elems * 8
        push.epoch = regions[0].data_ptr()
        pushes.append(push)
    lib = _abi.load()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)

    def push_gemv(m, a, src=0):  # the current stream at call time (graph capture uses a side stream)
        _abi.check(lib.wal_rvq_gemv_push(ctypes.byref(m.layer_struct()), a.data_ptr(), a.shape[0], a.stride(0),
                                         ctypes.byref(pushes[src]), _abi.stream_handle(DEV)), "push")

    def reduce():
        # every rank's words carry tag 1 after one push, so the wait returns at once;
        # the region's call count is reset so each replay finds the same tag
        _abi.check(lib.wal_tp_reduce_rmsnorm(regions[0].data_ptr() + 4096, tp, slot_elems, s.hidden,
                                             regions[0].data_ptr(), regions[0].data_ptr() + 1024, h.data_ptr(),
                                             h.stride(0), nw.data_ptr(), 1e-5, xo.data_ptr(), xo.stride(0), batch,
                                             s.hidden, status.data_ptr(), _abi.stream_handle(DEV)), "reduce")
        regions[0][:4].zero_()

    pos = context
    groups = {
        "qkv_gemv": lambda: qkv.gemv_into(x, yqkv),
        "rope_kv_append": lambda: rope_kv_append(yqkv, hq, hkv, hd, cos, sin, pos, q, kc, vc),
        "decode_attention": lambda: decode_attention(q, kc, vc, pos + 1, attn, ws),
        "o_push_gemv": lambda: push_gemv(o, attn),
        "reduce_rmsnorm": reduce,
        "gate_up_gemv": lambda: gu.gemv_into(x, ygu),
        "silu_mul": lambda: silu_mul(ygu, act),
        "down_push_gemv": lambda: push_gemv(down, act),
        "residual_rmsnorm_local": lambda: residual_rmsnorm(h, nw, 1e-5, xo),
        "call_count_reset": lambda: regions[0][:4].zero_(),  # part of reduce_rmsnorm above; subtract
    }
    # every sender's words of region 0 carry tag 1 before the reduction is timed;
    # one untimed reduction must find them (else the bounded wait reports it)
    for src in range(tp):
        push_gemv(down, act, src)
    reduce()
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError("exchange wait timed out")
    reps = 200
    out = {"case": "tp_breakdown", "tp": tp, "batch": batch, "context": context, "us": {}}
    for name, fn in groups.items():
        fn()
        torch.cuda.synchronize()
        probe = torch.cuda.CUDAGraph()  # a short replay first: a stuck wait costs 2 s, not 200 x 2 s
        with torch.cuda.graph(probe):
            for _ in range(3):
                fn()
        probe.replay()
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise RuntimeError(f"exchange wait timed out in {name}")
        del probe
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        out["us"][name] = round(e0.elapsed_time(e1) * 1e3 / reps, 3)
        del graph
    if int(status.item()) != 0:
        raise RuntimeError("exchange wait timed out")
    us = out["us"]
    us["reduce_rmsnorm"] = round(us["reduce_rmsnorm"] - us.pop("call_count_reset"), 3)
    per_layer = sum(v for k, v in us.items() if k != "residual_rmsnorm_local") + us["reduce_rmsnorm"]
    out["per_layer_us_sum"] = round(per_layer, 3)
    print(json.dumps(out))


def tp_breakdown_all() -> None:
    for tp in (1, 2, 4, 8):
        for batch in (1, 32):
            tp_breakdown(tp, batch)


CASES = {"cfg1_gemv": cfg1_gemv, "gemv_window": gemv_window, "idroute_mlp": idroute_mlp, "attention": attention,
         "prefill_gate_up": prefill_gate_up, "tp_breakdown": tp_breakdown_all}


def main(argv: list[str]) -> int:
    if len(argv) != 1 or argv[0] not in CASES:
        print(f"usage: python -m wal2026_b200.profile_cases {{{','.join(CASES)}}}", file=sys.stderr)
        return 2
    CASES[argv[0]]()
    torch.cuda.synchronize()
    print(f"{argv[0]}: ok")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
