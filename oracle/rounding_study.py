"""How far a decode that skips the second bf16 rounding lands from the reference (CPU study, test infrastructure).

The reference's bf16 weight is ``w = bf16(bf16(sum_s c_s) * bf16(rho))``
(``src/runtime.py:379-414``); the north star's output gate is
``max|y - y_ref| <= 2e-3 * ||y_ref||_inf`` against ``y_ref = x @ w^T``
accumulated in fp32.  A decode that keeps the first rounding (the stage sum,
free for one-stage tables) but applies ``bf16(rho)`` to the row's fp32 result
instead of to every weight would drop one multiply per weight pair.  This
script measures, over many seeds of the benchmark configurations, the error
of that variant against ``y_ref`` (float64 arithmetic; only the weight
rounding differs):

    python -m oracle.rounding_study cfg0 100
    python -m oracle.rounding_study cfg1 100
    python -m oracle.rounding_study qkv 30
"""
from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from wal2026_b200 import synthetic  # noqa: E402


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float64)


def _errors(wn: torch.Tensor, rho: torch.Tensor, K: int, seed: int, Ms) -> list[float]:
    """Relative max error of y = (x @ wn^T) * rho against x @ bf16(wn * rho)^T, per token count."""
    wref = _bf(wn * rho)
    out = []
    for M in Ms:
        x = synthetic.activations(M, K, seed=seed).double()
        yref = x @ wref.T
        yvar = (x @ wn.T) * rho.T
        out.append(float((yvar - yref).abs().max() / yref.abs().max()))
    return out


def cfg1_case(seed: int) -> list[float]:
    ri = synthetic.route_inputs(14336, 4096, seed=seed)
    ids = ri.route.long() * 256 + ri.code.long()
    wn = _bf(ri.codebooks.reshape(-1, 16).float())[ids].reshape(14336, 4096)  # one stage: bf16(c)
    return _errors(wn, _bf(ri.row_scale.float()), 4096, seed, (1, 8, 16))


def rvq_case(N: int, K: int, seed: int) -> list[float]:
    enc = synthetic.rvq_encoding(N, K, seed=seed)
    s = torch.zeros(N * (K // 8), 8, dtype=torch.float32)
    for ids, cb in zip(enc.stage_ids, enc.codebooks):
        s += cb.float()[ids.reshape(-1).long()]
    wn = _bf(s).reshape(N, K)  # first rounding of the fp32 stage sum
    return _errors(wn, _bf(enc.row_scale.float()), K, seed, (1, 4, 16))


CASES = {"cfg1": cfg1_case, "cfg0": lambda s: rvq_case(2048, 2048, s), "qkv": lambda s: rvq_case(6144, 4096, s)}


def main(argv: list[str]) -> int:
    which, n = argv[0], int(argv[1])
    torch.set_num_threads(max(1, torch.get_num_threads()))
    t0 = time.time()
    res = np.array([CASES[which](s) for s in range(n)])
    print(f"{which} seeds={n} max={res.max(0)} mean={res.mean(0)} p99={np.percentile(res, 99, axis=0)} "
          f"share_above_2e-3={(res > 2e-3).mean(0)} ({time.time() - t0:.0f} s)")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
