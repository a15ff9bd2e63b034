"""Seeded synthetic inputs for the benchmark configurations.

No public dataset or checkpoint is involved: every configuration is defined by
shapes and value distributions, drawn from a CPU ``torch.Generator`` in a fixed
order so the same seed gives the same bytes in the fixture generator, the
tests and the benchmark.

Configurations (the benchmark's own descriptions, restated):

* cfg0 - single Block-RVQ linear 2048x2048, d=8, R=2 stages of 256 entries,
  codes uniform, codebook stage 0 ~ N(0, 0.02), stage 1 ~ N(0, 0.005), fp16
  row scale ~ U(0.5, 1.5), activations bf16 ~ N(0, 1), M in {1, 4, 16};
* cfg1 - route-codebook linear 4096 -> 14336, d=16, a uint8 route over G=16
  codebooks drawn Zipf(s=1.1) plus a uniform uint8 code, codebooks
  [16, 256, 16] ~ N(0, 0.02), M in {1, 8, 16};
* Llama-shaped layers use the cfg0 distributions for every linear.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .block_vq import (
    BlockRVQEncoding,
    GroupedBlockRVQEncoding,
    make_plain_encoding,
    route_code_encoding,
    single_group,
)

CFG0_SHAPE = dict(N=2048, K=2048, d=8, R=2, C=256)
CFG1_SHAPE = dict(N=14336, K=4096, d=16, G=16, C=256)
ZIPF_S = 1.1


def _gen(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(int(seed))


def rvq_encoding(
    N: int,
    K: int,
    *,
    d: int = 8,
    R: int = 2,
    C: int = 256,
    seed: int = 0,
    stage_std: tuple[float, ...] = (0.02, 0.005),
) -> BlockRVQEncoding:
    """Plain R-stage encoding with the cfg0 distributions (draw order: codes, codebooks, scales)."""
    g = _gen(seed)
    B = -(-K // d)
    codes = torch.randint(0, C, (N, B, R), generator=g, dtype=torch.int64)
    books = []
    for r in range(R):
        std = stage_std[r] if r < len(stage_std) else stage_std[-1] / (4 ** (r - len(stage_std) + 1))
        books.append((torch.randn(C, d, generator=g) * std).to(torch.float16))
    rho = (torch.rand(N, 1, generator=g) + 0.5).to(torch.float16)
    id_dtype = torch.uint8 if C <= 256 else torch.int16
    stage_ids = [codes[:, :, r].to(id_dtype).contiguous() for r in range(R)]
    return make_plain_encoding(stage_ids, books, rho, in_features=K, block_size=d)


def zipf_probs(G: int, s: float = ZIPF_S) -> torch.Tensor:
    ranks = torch.arange(1, G + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    return p / p.sum()


@dataclass
class RouteInputs:
    route: torch.Tensor      # uint8 [N, B]
    code: torch.Tensor       # uint8 [N, B]
    codebooks: torch.Tensor  # fp16 [G, C, d]
    row_scale: torch.Tensor  # fp16 [N, 1]
    in_features: int

    def encoding(self) -> BlockRVQEncoding:
        return route_code_encoding(self.route, self.code, self.codebooks, self.row_scale,
                                   in_features=self.in_features)


def route_inputs(N: int, K: int, *, d: int = 16, G: int = 16, C: int = 256, seed: int = 1) -> RouteInputs:
    """cfg1 distributions (draw order: routes, codes, codebooks, scales)."""
    g = _gen(seed)
    B = -(-K // d)
    p = zipf_probs(G)
    route = torch.multinomial(p, N * B, replacement=True, generator=g).to(torch.uint8).view(N, B)
    code = torch.randint(0, C, (N, B), generator=g, dtype=torch.int64).to(torch.uint8)
    books = (torch.randn(G, C, d, generator=g) * 0.02).to(torch.float16)
    rho = (torch.rand(N, 1, generator=g) + 0.5).to(torch.float16)
    return RouteInputs(route.contiguous(), code.contiguous(), books.contiguous(), rho, K)


def activations(M: int, K: int, *, seed: int) -> torch.Tensor:
    """bf16 activations ~ N(0, 1) from their own generator (seed, M)."""
    g = _gen(seed * 1000 + M)
    return torch.randn(M, K, generator=g).to(torch.bfloat16)


def bias_vector(N: int, *, seed: int) -> torch.Tensor:
    g = _gen(seed * 7919 + 13)
    return (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)


def cfg0_encoding(seed: int = 0) -> GroupedBlockRVQEncoding:
    s = CFG0_SHAPE
    return single_group(rvq_encoding(s["N"], s["K"], d=s["d"], R=s["R"], C=s["C"], seed=seed))


def cfg1_inputs(seed: int = 1) -> RouteInputs:
    s = CFG1_SHAPE
    return route_inputs(s["N"], s["K"], d=s["d"], G=s["G"], C=s["C"], seed=seed)


def grouped_encoding(row_counts: list[int], K: int, *, d: int = 8, R: int = 2, C: int = 256,
                     seed: int = 0) -> GroupedBlockRVQEncoding:
    """Several row groups with independent codebooks (e.g. fused q/k/v)."""
    groups = []
    slices = []
    row0 = 0
    for i, n in enumerate(row_counts):
        groups.append(rvq_encoding(n, K, d=d, R=R, C=C, seed=seed * 101 + i))
        slices.append((row0, row0 + n))
        row0 += n
    return GroupedBlockRVQEncoding(groups=tuple(groups), row_slices=tuple(slices), original_shape=(row0, K))


@dataclass
class IDRouteInputs:
    """Constructor arguments of an ID-route linear (reference ``PackedIDRouteLinear``)."""

    ids: torch.Tensor         # int32 [N, K]
    codebook_w: torch.Tensor  # fp16 [routes, L]
    row_scale: torch.Tensor   # fp16 [N, 1]


def idroute_inputs(N: int, K: int, *, routes: int = 1536, L: int = 12, seed: int = 21) -> IDRouteInputs:
    """Seeded ID-route weight: uniform ids, fp16 route digits ~ N(0, 0.01), row scales ~ U(0.5, 1.5)."""
    g = _gen(seed)
    ids = torch.randint(0, routes, (N, K), generator=g, dtype=torch.int64).to(torch.int32)
    codebook_w = (torch.randn(routes, L, generator=g) * 0.01).to(torch.float16)
    rho = (torch.rand(N, 1, generator=g) + 0.5).to(torch.float16)
    return IDRouteInputs(ids, codebook_w, rho)

