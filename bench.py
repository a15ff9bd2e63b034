#!/usr/bin/env python3
"""Benchmark: route-codebook / Block-RVQ decode gather-GEMV throughput on B200.

Workload (one "step"): the decode GEMV (M tokens, default 1) of config 1 -
route-codebook linear 4096 -> 14336, d=16, uint8 route over G=16 codebooks
(Zipf s=1.1) plus uint8 code, fp16 codebooks [16, 256, 16], fp16 row scales -
over `--instances` distinct seeded weight instances (default 32, ~241 MB of
compressed weight, i.e. larger than the 126 MB L2), so every GEMV streams its
ids from HBM.  The metric is GB/s of algorithmic (compressed) bytes:
ids + codebooks + row scales + x + y per GEMV, each counted once.

Arms:
  default            this package's CUDA path (C ABI), one CUDA graph per step;
  --impl reference   the reference's dequantise-then-matmul algorithm on the
                     host cores (C restatement in oracle/, all threads), same
                     metric and config, rank 0 only.

Multi-GPU (torchrun): every rank runs its own instances (weak scaling, no
collective on the data path); the time is the max over ranks.

Also reported in the same JSON line (BASELINE's second metric and configs 0, 2, 3, 4):
  gemv_configs (N = 1) config 0 (Block-RVQ 2048 x 2048, d=8, R=2) at M = 1/4/16
              over 256 distinct instances, and config 1 at M = 8/16, GB/s of
              algorithmic bytes with a roofline against the measured HBM copy;
  decode_8b   Llama-3-8B-shaped stack (random init, every projection Block-RVQ
              d=8, R=2, 256 entries; dense bf16 lm_head), one CUDA graph per
              decode step at a 2048-token context, tensor-parallel over all
              N GPUs (NVLink push exchange after the row-parallel linears),
              next to the same stack with dense bf16 cuBLAS projections (same
              push exchange; at N > 1 also with an NCCL all-reduce); at N > 1
              the logits of one sharded step against the unsharded stack;
  decode_1b   config 2: the Llama-3.2-1B-shaped stack at batch 1/16 on a
              512-token context, same arms;
  decode_70b  config 4: the Llama-3-70B-shaped stack at batch 1/16/64 on a
              4096-token context, same arms; configurations that do not fit
              a GPU's memory at this N are listed as skipped;
  prefill_8b  (N = 1) the stack's 128 projection GEMMs at M = 2048 tokens on
              the tcgen05 decode-to-shared-memory GEMM, TFLOP/s against the
              measured bf16 peak, next to cuBLAS on the same shapes;
  idroute_gemv (N = 1) the ID-route linear (reference PackedIDRouteLinear:
              an int16 id per weight into fp16 route sums) on the 8B MLP
              shape, GB/s against the measured HBM bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_OUT, K_IN, D, G = 14336, 4096, 16, 16
METRIC = "RVQ gather-GEMV GB/s (% of 8 TB/s HBM); 8B decode tok/s at 1/2/4/8 B200"
UNIT = "GB/s"
NOMINAL_HBM_GBS = 8000.0
# DRAM bytes per launch of rvq_gemv_kernel on this workload (one cfg1 instance, M = 1):
# dram__bytes_read.sum + dram__bytes_write.sum from an ncu capture of
# `python -m wal2026_b200.profile_cases cfg1_gemv`.
NCU_TRAFFIC_BYTES = 7532288


def algorithmic_bytes(M: int) -> int:
    blocks = -(-K_IN // D)
    ids = N_OUT * blocks * 2  # route + code per unit
    books = G * 256 * D * 2
    rho = N_OUT * 2
    return ids + books + rho + 2 * M * K_IN + 2 * M * N_OUT


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons in the background (no settings are changed)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu_index = gpu_index
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        rows = []
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), float(parts[3]), parts[4:8]))
            except ValueError:
                continue
        if not rows:
            return None
        busy = [r for r in rows if r[3] > 0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i, v in enumerate(r[4]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in busy), "sm_max_mhz": max(r[1] for r in busy),
                "reasons": reasons, "samples": len(busy), "power_w_max": max(r[2] for r in busy)}


def make_instances(n: int, seed0: int, device: torch.device):
    from wal2026_b200 import synthetic
    from wal2026_b200.runtime import RouteCodebookLinear

    mods = []
    for i in range(n):
        inp = synthetic.route_inputs(N_OUT, K_IN, d=D, G=G, seed=seed0 + i)
        mods.append(RouteCodebookLinear.from_routes(inp.route, inp.code, inp.codebooks, inp.row_scale,
                                                    in_features=K_IN).to(device))
    return mods


def cpu_oracle_sample(M: int, rows: int, min_seconds: float, min_reps: int = 2):
    """Time the reference algorithm (C restatement, all host threads) on `rows` rows of cfg1."""
    from oracle import c_oracle  # CPU baseline leg only
    from oracle import rvq_oracle as orc
    from wal2026_b200 import synthetic

    inp = synthetic.route_inputs(N_OUT, K_IN, d=D, G=G, seed=1)
    enc = inp.encoding()
    g = orc.groups_from_encoding(enc)[0]
    sample = {"stage_ids": [g["stage_ids"][0][:rows]], "codebooks": g["codebooks"], "row_scale": g["row_scale"][:rows]}
    x = synthetic.activations(M, K_IN, seed=1).view(torch.int16).numpy().view(np.uint16)
    threads = c_oracle.max_threads()
    c_oracle.forward(x, [sample], K_IN, threads=threads)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        c_oracle.forward(x, [sample], K_IN, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= min_seconds:
            break
    blocks = -(-K_IN // D)
    per_rep = rows * (blocks * 2 + 2 + 2 * M) + G * 256 * D * 2 + 2 * M * K_IN
    return per_rep * reps / el / 1e9, threads, reps, el


def run_reference(args) -> None:
    """Reference arm: the reference algorithm on the host cores, one row-sample forward per step."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle import c_oracle  # the reference arm runs the CPU restatement

    rows = args.ref_rows
    threads = c_oracle.max_threads()
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        _ref_step(args.M, rows, threads)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    blocks = -(-K_IN // D)
    per_step = rows * (blocks * 2 + 2 + 2 * args.M) + G * 256 * D * 2 + 2 * args.M * K_IN
    total = sum(times)
    value = per_step * len(times) / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / len(times), 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(args),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{rows} of {N_OUT} rows of one cfg1 GEMV per step (dequantise-then-matmul, "
                                   f"C restatement of the reference, {threads} threads)"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


_REF_CACHE: dict = {}


def _ref_step(M: int, rows: int, threads: int) -> None:
    from oracle import c_oracle
    from oracle import rvq_oracle as orc
    from wal2026_b200 import synthetic

    key = (M, rows)
    if key not in _REF_CACHE:
        inp = synthetic.route_inputs(N_OUT, K_IN, d=D, G=G, seed=1)
        g = orc.groups_from_encoding(inp.encoding())[0]
        sample = {"stage_ids": [g["stage_ids"][0][:rows]], "codebooks": g["codebooks"],
                  "row_scale": g["row_scale"][:rows]}
        x = synthetic.activations(M, K_IN, seed=1).view(torch.int16).numpy().view(np.uint16)
        _REF_CACHE[key] = (sample, x)
    sample, x = _REF_CACHE[key]
    c_oracle.forward(x, [sample], K_IN, threads=threads)


def _config(args) -> dict:
    return {
        "workload": f"cfg1 route-codebook linear {K_IN}->{N_OUT}, d={D}, G={G} Zipf(1.1) routes + uint8 codes, "
                    f"M={args.M} decode GEMV",
        "M": args.M, "N": N_OUT, "K": K_IN, "instances": args.instances,
        "bytes_per_gemv": algorithmic_bytes(args.M),
        "l2": f"inputs larger than L2: {args.instances} distinct weight instances "
              f"({args.instances * algorithmic_bytes(args.M) / 1e6:.0f} MB) per step",
    }


def _decode_bytes_per_rank(shape, kind: str, batch: int, context: int, world: int) -> int:
    """Device bytes one rank needs for a decode stack of this shape (weights, embeddings, KV cache, slack)."""
    hd = shape.head_dim
    per_layer = (shape.heads * hd + 2 * shape.kv_heads * hd) * shape.hidden + shape.heads * hd * shape.hidden \
        + 3 * shape.mlp * shape.hidden
    weights = shape.layers * per_layer * (2.0 if kind.startswith("dense") else 0.25) / world
    embed = shape.vocab * shape.hidden * 2 * (1 + 1.0 / world)
    kv = shape.layers * 2 * batch * (shape.kv_heads // world) * (context + 1) * hd * 2
    draw = 2 * shape.mlp * shape.hidden * 6  # one full gate/up layer drawn before sharding (fp32 + bf16)
    return int(weights + embed + kv + draw + 4e9)


DECODE_LEGS = {
    # which: (model name, batches argument, context argument)
    "1b": ("Llama-3.2-1B", "decode1b_batches", "context1b"),
    "8b": ("Llama-3-8B", "decode_batches", "context"),
    "70b": ("Llama-3-70B", "decode70_batches", "context70"),
}


def _tp_step_logits(st, shape, dev, context: int, tokens, push: bool) -> torch.Tensor:
    st.allocate_cache(int(tokens.shape[0]), context + 1, consistent=True, seed=19)
    cos, sin = st.rope_tables(context)
    if push:
        st.enable_push_exchange(int(tokens.shape[0]))
    logits = st.decode_step_fused(tokens, context, cos, sin, exchange="push" if push else "nccl").float()
    torch.cuda.synchronize()
    st.k_cache, st.v_cache = [], []
    return logits


def tp_logits_check(st, shape, which: str, rank: int, world: int, dev: torch.device, context: int) -> dict | None:
    """One tensor-parallel decode step's logits against the unsharded stack (rank 0 reports).

    Every rank holds a shard of the same seeded model and a slice of the same
    cache, so the sharded step (push exchange) equals the single-GPU step up to
    the order of the fp32 partial sums, whose bf16 roundings then propagate
    through the layers.  Reported for the whole stack and, to show the
    per-layer size of that effect, for a one-layer stack of the same shape.
    """
    import dataclasses

    import torch.distributed as dist

    from wal2026_b200.llama import TPContext, rvq_llama

    gen = torch.Generator(device=dev).manual_seed(17)
    tokens = torch.randint(0, shape.vocab, (1,), device=dev, generator=gen)
    res = {}
    one = dataclasses.replace(shape, layers=1)
    tp = TPContext(rank, world, dist.group.WORLD)
    for label, shp, stack in (("stack", shape, st), ("one_layer", one, None)):
        own = stack if stack is not None else rvq_llama(shp, device=dev, seed=0, tp=tp)
        logits = _tp_step_logits(own, shp, dev, context, tokens, push=True)
        if stack is None:
            own.close()
            del own
        if rank == 0:
            full = rvq_llama(shp, device=dev, seed=0)
            ref = _tp_step_logits(full, shp, dev, context, tokens, push=False)
            del full
            torch.cuda.empty_cache()
            res[label] = {
                "max_rel_err": round(float((logits - ref).abs().max() / ref.abs().max()), 6),
                "cosine": round(float(torch.nn.functional.cosine_similarity(logits, ref, dim=-1).min()), 6),
                "top1_agree": bool((logits.argmax(-1) == ref.argmax(-1)).all()),
            }
        dist.barrier()
    return res if rank == 0 else None


def run_decode(args, rank: int, world: int, dev: torch.device, which: str = "8b") -> dict:
    """Llama-shaped decode tok/s, tensor-parallel over every rank (all ranks call this together)."""
    import torch.distributed as dist

    from wal2026_b200.llama import SHAPES, TPContext, dense_llama, rvq_llama, time_decode

    shape = SHAPES[which]
    tp = TPContext(rank, world, dist.group.WORLD if world > 1 else None)
    name, batches_arg, context_arg = DECODE_LEGS[which]
    batches = [int(b) for b in getattr(args, batches_arg).split(",") if b]
    context = int(getattr(args, context_arg))
    total = torch.cuda.get_device_properties(dev).total_memory
    exch = "nvlink push (tagged words)" if world > 1 else "none"
    out = {"model": f"{name} shape ({shape.layers} layers, hidden {shape.hidden}, MLP {shape.mlp}, "
                    f"{shape.heads} q / {shape.kv_heads} kv heads, vocab {shape.vocab}), random init; "
                    "q/k/v/o/gate/up/down Block-RVQ d=8 R=2 256 entries; lm_head dense bf16",
           "context": context, "tp": world, "exchange": exch,
           "graph": "one CUDA graph per decode step", "steps": args.decode_steps}
    # the dense comparator runs the same push exchange as the RVQ stack (a
    # separate push of the cuBLAS output) and, under tensor parallelism, also
    # the NCCL all-reduce, so the speed-up compares linears, not exchanges
    arms = [("rvq", rvq_llama, "push"), ("dense_bf16_cublas", dense_llama, "push")]
    if world > 1:
        arms.append(("dense_bf16_cublas_nccl", dense_llama, "nccl"))
    for kind, ctor, exchange in arms:
        if kind.startswith("dense") and not args.dense:
            continue
        dkind = "dense" if kind.startswith("dense") else "rvq"
        fits = [b for b in batches if _decode_bytes_per_rank(shape, dkind, b, context, world) < 0.85 * total]
        res = {str(b): {"skipped": f"needs ~{_decode_bytes_per_rank(shape, dkind, b, context, world) / 1e9:.0f} GB "
                                   f"per GPU at tp={world}"} for b in batches if b not in fits}
        if fits:
            st = ctor(shape, device=dev, seed=0, tp=tp)
            for b in fits:
                r = time_decode(st, b, context, steps=args.decode_steps, warmup=3, fused=True, exchange=exchange)
                res[str(b)] = {"tok_s": round(r["tok_s"], 1), "ms_per_step": round(r["ms_per_step"], 4)}
                st.k_cache, st.v_cache = [], []
                st._bufs.clear()
                torch.cuda.empty_cache()
            if kind == "rvq":
                out["rvq_projection_bytes_per_rank"] = st.linear_bytes()
                if world > 1 and args.tp_check:
                    out["tp_logits_vs_unsharded"] = tp_logits_check(st, shape, which, rank, world, dev, context)
            st.close()
            del st
            torch.cuda.empty_cache()
        out[kind] = {b: res[b] for b in map(str, batches)}
    if "dense_bf16_cublas" in out:
        out["rvq_speedup_vs_dense"] = {
            b: round(out["rvq"][b]["tok_s"] / out["dense_bf16_cublas"][b]["tok_s"], 3)
            for b in out["rvq"] if "tok_s" in out["rvq"][b] and "tok_s" in out["dense_bf16_cublas"][b]}
    return out


def _gemv_line(mods, M: int, K: int, reps: int, bytes_per: int, peak: float, dev: torch.device) -> dict:
    """GB/s of one GEMV shape over distinct instances (inputs larger than L2), graph replay, CUDA events."""
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    y = torch.empty(M, mods[0].out_features, device=dev, dtype=torch.bfloat16)
    for m in mods:
        m.gemv_into(x, y)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for m in mods:
            m.gemv_into(x, y)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * len(mods))
    gbs = bytes_per / (us * 1e-6) / 1e9
    del g
    return {"M": M, "us_per_gemv": round(us, 3), "gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "algorithmic_bytes_per_launch": bytes_per},
            "gpu_launches": reps * len(mods)}


def run_gemv_configs(args, dev: torch.device, peaks: dict, cfg1_mods) -> dict:
    """cfg0 (2048 x 2048, d=8, R=2) at M = 1/4/16 and cfg1 at M = 8/16 (the headline is cfg1 at M = 1)."""
    from wal2026_b200.runtime import PackedGroupedBlockRVQLinear

    peak = float(peaks.get("hbm_gbs") or 6650.0)
    out = {"peak_source": "measured hbm_gbs" if peaks.get("hbm_gbs") else "fallback"}
    N, K, d, R = 2048, 2048, 8, 2
    gen = torch.Generator(device=dev).manual_seed(23)
    mods = [PackedGroupedBlockRVQLinear.random([N], K, block_size=d, num_stages=R, generator=gen, device=dev)
            for _ in range(args.cfg0_instances)]
    lines = []
    for M in (1, 4, 16):
        nbytes = N * (K // d) * R + R * 256 * d * 2 + 2 * N + 2 * M * K + 2 * M * N
        lines.append(_gemv_line(mods, M, K, 20, nbytes, peak, dev))
    out["cfg0"] = {"workload": f"Block-RVQ linear {K}->{N}, d={d}, R={R}, 256 entries (cfg0 distributions), "
                               f"{len(mods)} distinct instances ({len(mods) * N * K * R // d / 1e6:.0f} MB of ids, "
                               "larger than L2) per graph", "lines": lines}
    del mods
    lines = []
    for M in (8, 16):
        lines.append(_gemv_line(cfg1_mods, M, K_IN, 20, algorithmic_bytes(M), peak, dev))
    out["cfg1"] = {"workload": f"cfg1 route-codebook linear {K_IN}->{N_OUT}, {len(cfg1_mods)} instances per graph",
                   "lines": lines}
    torch.cuda.empty_cache()
    return out


def run_prefill(args, dev: torch.device, peaks: dict) -> dict:
    """8B-shaped prefill GEMMs (M = 2048) on the tcgen05 path, one CUDA graph of all 128 projections."""
    import torch.nn.functional as F

    from wal2026_b200.llama import LLAMA_8B, rvq_llama

    M = args.prefill_tokens
    st = rvq_llama(LLAMA_8B, device=dev, seed=0)
    lins = [getattr(layer, n) for layer in st.layers for n in ("qkv", "o", "gate_up", "down")]
    xs = {k: torch.randn(M, k, device=dev).to(torch.bfloat16) for k in {lin.in_features for lin in lins}}
    ys = {n: torch.empty(M, n, device=dev, dtype=torch.bfloat16) for n in {lin.out_features for lin in lins}}
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def run():
        for lin in lins:
            if not lin.gemm_into(xs[lin.in_features], ys[lin.out_features], status):
                raise RuntimeError("prefill GEMM path does not cover this layer")

    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.prefill_steps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError("prefill GEMM reported a pipeline timeout")
    ms = e0.elapsed_time(e1) / args.prefill_steps
    flops = sum(2.0 * M * lin.out_features * lin.in_features for lin in lins)
    tflops = flops / (ms / 1e3) / 1e12
    del g
    # cuBLAS bf16 on the same shapes (one layer's four dense weights, repeated for 32 layers)
    dense = None
    if args.dense:
        ws = [torch.randn(lin.out_features, lin.in_features, device=dev).to(torch.bfloat16) for lin in lins[:4]]
        for w in ws:
            F.linear(xs[w.shape[1]], w)
        torch.cuda.synchronize()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for _ in range(args.prefill_steps):
            for _layer in range(LLAMA_8B.layers):
                for w in ws:
                    F.linear(xs[w.shape[1]], w)
        d1.record(stream)
        torch.cuda.synchronize()
        dms = d0.elapsed_time(d1) / args.prefill_steps
        dense = {"ms_per_step": round(dms, 3), "tflops": round(flops / (dms / 1e3) / 1e12, 1)}
        del ws
    peak = float(peaks.get("bf16_tflops_sustained") or 1400.0)
    src = "measured bf16_tflops_sustained" if peaks.get("bf16_tflops_sustained") else "fallback"
    launches = len(lins) * args.prefill_steps
    del st, lins
    torch.cuda.empty_cache()
    return {"workload": f"Llama-3-8B-shaped stack, 128 projection GEMMs at M={M} tokens (x bf16, y bf16)",
            "ms_per_step": round(ms, 3), "tokens_per_s": round(M / (ms / 1e3), 1), "tflops": round(tflops, 1),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4), "peak_source": src, "kernel": "rvq_gemm_pair_kernel"},
            "gpu_launches": launches, "dense_bf16_cublas": dense}


def run_idroute(args, dev: torch.device, peaks: dict) -> dict:
    """ID-route GEMV (reference PackedIDRouteLinear, 2 bytes of ids per weight) on the 8B MLP shape, M = 1."""
    from wal2026_b200.idroute import PackedIDRouteLinear

    N, K, routes, M = N_OUT, K_IN, 1536, args.M
    gen = torch.Generator(device=dev).manual_seed(5)
    mods = [PackedIDRouteLinear.random(N, K, routes=routes, generator=gen, device=dev) for _ in range(4)]
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    for m in mods:
        m.gemv_into(x, y)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for m in mods:
            m.gemv_into(x, y)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(5, args.steps)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * len(mods))
    nbytes = N * K * 2 + routes * 2 + N * 2 + 2 * M * K + 2 * M * N
    gbs = nbytes / (us * 1e-6) / 1e9
    peak = float(peaks.get("hbm_gbs") or 6650.0)
    del g, mods
    torch.cuda.empty_cache()
    return {"workload": f"ID-route linear {K}->{N}, int16 id per weight into {routes} fp16 route sums, M={M}, "
                        f"4 instances ({4 * N * K * 2 / 1e6:.0f} MB, larger than L2) per graph",
            "us_per_gemv": round(us, 3), "gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_source": "measured hbm_gbs" if peaks.get("hbm_gbs")
                         else "fallback", "kernel": "idroute_gemv_kernel", "algorithmic_bytes_per_launch": nbytes}}


def run_ours(args) -> None:
    import torch.distributed as dist

    from wal2026_b200 import _abi

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    _abi.load()
    mods = make_instances(args.instances, 1 + 1000 * rank, dev)
    from wal2026_b200 import synthetic

    x = synthetic.activations(args.M, K_IN, seed=1).to(dev)
    y = torch.empty((args.M, N_OUT), device=dev, dtype=torch.bfloat16)
    for m in mods:  # first calls set kernel attributes outside graph capture
        m.gemv_into(x, y)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for m in mods:
            m.gemv_into(x, y)
    stream = torch.cuda.current_stream()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                           else int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local]))
    # untimed soak so the clock sampler sees the GPU under this load
    t_end = time.time() + args.soak
    while time.time() < t_end:
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    launches = args.steps * len(mods)
    bytes_per = algorithmic_bytes(args.M)
    value = world * bytes_per * launches / (ms / 1e3) / 1e9
    per_launch_s = (ms / 1e3) / launches
    achieved = bytes_per / per_launch_s / 1e9

    # end to end through the public call with host buffers (pinned), copies inside the timed region:
    # every step copies its input x to the device, runs the instances' GEMVs
    # one C-ABI call each (Python loop, no graph) and reads all their outputs back
    xh = synthetic.activations(args.M, K_IN, seed=1).pin_memory()
    yh = torch.empty((len(mods), args.M, N_OUT), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(xh, device=dev)
    yd = torch.empty((len(mods), args.M, N_OUT), dtype=torch.bfloat16, device=dev)
    e2e_steps = max(1, min(args.steps, 20))

    def e2e_step():
        xd.copy_(xh, non_blocking=True)
        for i, m in enumerate(mods):
            m.gemv_into(xd, yd[i])
        yh.copy_(yd, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * bytes_per * e2e_steps * len(mods) / (e2e_ms / 1e3) / 1e9

    # dense bf16 cuBLAS GEMV on the same shape (comparison only)
    dense = None
    if args.dense and rank == 0:
        ws = [torch.randn(N_OUT, K_IN, device=dev, dtype=torch.bfloat16) for _ in range(min(8, args.instances))]
        for w in ws:
            torch.nn.functional.linear(x, w)
        torch.cuda.synchronize()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        d0.record(stream)
        for _ in range(reps):
            for w in ws:
                torch.nn.functional.linear(x, w)
        d1.record(stream)
        torch.cuda.synchronize()
        dms = d0.elapsed_time(d1) / (reps * len(ws))
        dense = {"ms_per_gemv": round(dms, 5), "weight_bytes": N_OUT * K_IN * 2,
                 "gbs_dense_bytes": round(N_OUT * K_IN * 2 / (dms / 1e3) / 1e9, 1),
                 "rvq_speedup": round(dms / (per_launch_s * 1e3), 3)}
        del ws

    peaks = measured_peaks()
    gemv_cfgs = run_gemv_configs(args, dev, peaks, mods) if (args.gemv_configs and world == 1) else None
    decode = run_decode(args, rank, world, dev) if args.decode else None
    decode1b = run_decode(args, rank, world, dev, "1b") if args.decode_1b else None
    decode70 = run_decode(args, rank, world, dev, "70b") if args.decode_70b else None
    # the ID-route leg runs before the prefill leg, whose sustained tensor work
    # leaves the GPU at its power cap for a while afterwards
    idroute = run_idroute(args, dev, peaks) if (args.idroute and world == 1) else None
    prefill = run_prefill(args, dev, peaks) if (args.prefill and world == 1) else None
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = float(peak or 6650.0)
    out = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            gbs, threads, reps, el = cpu_oracle_sample(args.M, args.ref_rows, args.cpu_seconds)
            cpu = {"value": round(gbs, 4), "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"{args.ref_rows} of {N_OUT} rows of a cfg1 GEMV x {reps} reps ({el:.1f} s), "
                             f"C restatement of the reference's dequantise-then-matmul"}
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _config(args),
            "pct_of_nominal_8tbs": round(100.0 * value / world / NOMINAL_HBM_GBS, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_src} hbm_gbs",
                         "traffic": NCU_TRAFFIC_BYTES,
                         "kernel": "rvq_gemv_kernel", "algorithmic_bytes_per_launch": bytes_per,
                         "avg_launch_us": round(per_launch_s * 1e6, 3)},
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": xh.numel() * 2,
                    "d2h_bytes_per_step": yh.numel() * 2,
                    "note": "per step: pinned H2D of x, one C-ABI GEMV per instance (Python loop, no graph), "
                            "D2H of every instance's y"},
            "gpu_launches": launches,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "dense_bf16_cublas": dense,
            "gemv_configs": gemv_cfgs,
            "decode_8b": decode,
            "decode_1b": decode1b,
            "decode_70b": decode70,
            "prefill_8b": prefill,
            "idroute_gemv": idroute,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        del graph
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--instances", type=int, default=32)
    ap.add_argument("--soak", type=float, default=1.5)
    ap.add_argument("--ref-rows", type=int, default=2048)
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--dense", type=int, default=1)
    ap.add_argument("--decode", type=int, default=1, help="also time the 8B-shaped decode step")
    ap.add_argument("--decode-batches", default="1,8,32")
    ap.add_argument("--decode-steps", type=int, default=20)
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--decode-70b", type=int, default=1, help="also time the 70B-shaped decode step (config 4)")
    ap.add_argument("--decode-1b", type=int, default=1, help="also time the 1B-shaped decode step (config 2)")
    ap.add_argument("--decode1b-batches", default="1,16")
    ap.add_argument("--context1b", type=int, default=512)
    ap.add_argument("--tp-check", type=int, default=1,
                    help="at N > 1, compare one tensor-parallel decode step's logits with the unsharded stack")
    ap.add_argument("--gemv-configs", type=int, default=1, help="also time cfg0 M=1/4/16 and cfg1 M=8/16 (N = 1)")
    ap.add_argument("--cfg0-instances", type=int, default=256)
    ap.add_argument("--decode70-batches", default="1,16,64")
    ap.add_argument("--context70", type=int, default=4096)
    ap.add_argument("--prefill", type=int, default=1, help="also time the 8B-shaped prefill GEMMs (N = 1)")
    ap.add_argument("--prefill-tokens", type=int, default=2048)
    ap.add_argument("--prefill-steps", type=int, default=5)
    ap.add_argument("--idroute", type=int, default=1, help="also time the ID-route GEMV (N = 1)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
