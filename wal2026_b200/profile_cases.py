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


CASES = {"cfg1_gemv": cfg1_gemv, "gemv_window": gemv_window, "idroute_mlp": idroute_mlp, "attention": attention,
         "prefill_gate_up": prefill_gate_up}


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
