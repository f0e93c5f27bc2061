"""bench.py's output contract, on the CPU: the reference arm (the
reference's host attention algorithm on the host cores) prints one JSON line
with the keys the driver reads; non-zero ranks of a torchrun launch exit 0
without work; the helpers that build the line follow the metric's formula.
(The engine arm needs a GPU and is covered by the -m gpu runs.)
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def run_bench(*args, env=None):
    e = dict(os.environ, **(env or {}))
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                          text=True, timeout=600, cwd=ROOT, env=e)


def test_reference_arm_prints_one_contract_line(oracle_mod):
    r = run_bench("--impl", "reference", "--steps", "2", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "TFLOP/s"
    assert d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 2 and d["warmup"] == 1 and d["value"] > 0
    assert d["config"]["S"] == 4096 and d["config"]["D"] == 128 and d["config"]["H"] == 16
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_runs_on_rank_0_only():
    r = run_bench("--impl", "reference", "--steps", "1", "--warmup", "0",
                  env={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_metric_formula_and_workloads():
    # 4 * B * H * S^2 * D per launch; units = B * H
    assert bench.flops(16, 4096, 128) == 4.0 * 16 * 4096 * 4096 * 128
    w = bench.WORKLOADS
    assert (w["c2"]["B"], w["c2"]["H"], w["c2"]["S"], w["c2"]["D"]) == (1, 16, 4096, 128)
    assert (w["c3"]["D"], w["c4"]["dtype"], w["c5"]["S"]) == (64, "bf16", 32768)
    assert w["c5"]["sigma"] == 0.5 and w["c2"]["scaling"] == "weak"
    assert w["c4"]["scaling"] == w["c5"]["scaling"] == "strong"


@pytest.mark.parametrize("wl,n,B", [("c2", 1, 1), ("c2", 4, 4), ("c4", 8, 8)])
def test_config_names_the_workload(wl, n, B):
    ns = type("A", (), {"bm": 256, "bn": 128, "seed": 1234})()
    cfg = bench.config_of(wl, ns, n)
    assert cfg["workload"].startswith(wl.upper()) and cfg["B"] == B
    assert cfg["causal"] is False and cfg["accumulate"] == "fp32"


def test_peaks_read_the_measured_file_or_fall_back():
    burst, sustained, kind = bench.peaks()
    assert kind in ("measured", "fallback")
    assert burst > sustained > 0
