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
# DRAM bytes per launch of rvq_gemv_kernel on this workload (one cfg1 instance, M = 1), from the
# ncu capture summarised in profiles/rvq_gemv_cfg1_m1.md: dram__bytes_read.sum + dram__bytes_write.sum.
NCU_TRAFFIC_BYTES = 7553536


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

    # end to end through the public call with host buffers (pinned), copies inside the timed region
    xh = synthetic.activations(args.M, K_IN, seed=1).pin_memory()
    yh = torch.empty((args.M, N_OUT), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(xh, device=dev)
    e2e_steps = max(1, min(args.steps, 20))
    for _ in range(2):
        for m in mods:
            xd.copy_(xh, non_blocking=True)
            m.gemv_into(xd, y)
            yh.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        for m in mods:
            xd.copy_(xh, non_blocking=True)
            m.gemv_into(xd, y)
            yh.copy_(y, non_blocking=True)
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
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": xh.numel() * 2 * len(mods),
                    "d2h_bytes_per_step": yh.numel() * 2 * len(mods),
                    "note": "per instance: pinned H2D of x, C-ABI GEMV, D2H of y; Python loop, no graph"},
            "gpu_launches": launches,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "dense_bf16_cublas": dense,
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
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
