"""bench.py's reference arm runs on the host cores (no GPU): its one JSON line keeps the driver's
contract, and under a multi-rank launch only rank 0 prints it."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    env.pop("CUDA_VISIBLE_DEVICES", None)
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "c1",
                           "--steps", "2", "--warmup", "1"], capture_output=True, text=True, cwd=ROOT, env=env,
                          timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    return [line for line in proc.stdout.splitlines() if line.strip()]


def test_reference_arm_prints_one_contract_line():
    lines = _run({"RANK": "0"})
    assert len(lines) == 1
    rec = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["impl"] == "reference" and rec["steps"] == 2 and rec["warmup"] == 1
    assert rec["value"] > 0 and rec["higher_is_better"] is True and rec["config"]["workload"] == "c1"
    cpu = rec["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == rec["value"] and cpu["sample"]
    assert rec["e2e"] == {"value": rec["value"], "unit": rec["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    assert _run({"RANK": "1", "WORLD_SIZE": "2"}) == []
