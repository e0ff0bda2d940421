"""bench.py's reference arm (the reference's CPU algorithm on host cores) keeps
the benchmark contract on a machine without a GPU: one JSON line from rank 0,
nothing from the other ranks."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench(*args, env=None):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, env={**os.environ, **(env or {})}, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    res = _bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert res.returncode == 0, res.stderr
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["value"] > 0
    assert line["higher_is_better"] is True and line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 3
    assert line["ms_per_step"] > 0 and line["data"] == "synthetic" and "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    res = _bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3",
                 env={"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr
    assert res.stdout.strip() == ""
