"""bench.py's reference arm (`--impl reference`), which needs no GPU: the oracle's restatement of the reference's CPU
decode timed on the host's cores, printed as one JSON line with the repo arm's metric and workload, a `cpu_baseline`
describing the run and an `e2e` that moves no bytes. Under torchrun only rank 0 runs it; the other ranks exit 0
without printing."""
import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_arm(env_extra):
    env = dict(os.environ, **env_extra)
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    return [line for line in p.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    lines = run_arm({"RANK": "0", "WORLD_SIZE": "1"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["config"]["workload"] == bench.DECODE_WORKLOAD
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    assert run_arm({"RANK": "1", "WORLD_SIZE": "2"}) == []
