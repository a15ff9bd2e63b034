"""bench.py's reference arm (the reference algorithm on the host cores) keeps the JSON contract.

Runs on the CPU: a tiny row sample of the config-1 GEMV through the C
restatement of the reference, as `bench.py --impl reference` does at full
size on the GPU box.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env: dict[str, str]) -> subprocess.CompletedProcess:
    env = dict(os.environ, **extra_env)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                           "--warmup", "3", "--ref-rows", "64"], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    res = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] >= 3 and d["n_gpus"] == 1
    assert d["metric"].startswith("RVQ gather-GEMV GB/s")
    assert "workload" in d["config"]
    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert not [l for l in res.stdout.splitlines() if l.startswith("{")]
