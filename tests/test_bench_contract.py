"""The bench's output contract, on the CPU: the reference arm's JSON line (the arm the driver runs
beside ours) and the headline metric's name, which must be BASELINE.json's."""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_module", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_headline_metric_is_baselines():
    bench = load_bench()
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        baseline = json.load(f)
    assert bench.metric_for("1024") == baseline["metric"] == bench.METRIC
    assert "@512²" in bench.metric_for("512") and "S=1536" in bench.metric_for("512")
    assert "@2048²" in bench.metric_for("2048") and "S=16896" in bench.metric_for("2048")


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "512",
                           "--steps", "1", "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip()]
    line = json.loads(lines[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == load_bench().metric_for("512")
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    # the median of at least 20 timed runs after at least 3 warm-ups, whatever --steps/--warmup ask for
    assert line["value"] > 0 and line["n_gpus"] == 1 and line["steps"] == 20 and line["warmup"] == 3
    assert line["ms_per_step"] > 0 and "median of 20 runs" in line["cpu_baseline"]["sample"]
    assert line["config"]["seq_len"] == 1536 and line["config"]["heads"] == 24
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
