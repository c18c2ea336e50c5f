"""The reference arm of bench.py (the CPU port of the reference's operators)
prints the one JSON line the benchmark contract asks for, on rank 0 only.

Runs on the CPU: a tiny workload (one request, 16 cached keys, one sampled
layer, no warm-up), so the numbers are meaningless and only the line's shape
is checked.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
ARGS = ["--impl", "reference", "--batch", "1", "--kv-len", "16", "--steps", "1", "--warmup", "0"]


def _run(extra_env):
    env = dict(os.environ, OPENBLAS_NUM_THREADS="4", OMP_NUM_THREADS="4", **extra_env)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE"):
        if k not in extra_env:
            env.pop(k, None)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *ARGS], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = _run({})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert d["metric"] == baseline["metric"]
    assert d["impl"] == "reference"
    assert d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["scaling"] == "weak" and d["vs_baseline"] is None and d["data"] == "synthetic"
    assert d["config"]["batch_per_gpu"] == 1 and d["config"]["kv_len"] == 16
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    r = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
