"""bench.py's reference arm runs on the host (no GPU) and prints one JSON line with the keys the
contract asks for: the metric and unit of the workload, `impl: reference`, a `cpu_baseline`
describing the run, and an `e2e` object with zero transfer bytes."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.join(os.path.dirname(__file__), "..")


@pytest.mark.parametrize("config,unit", [("small-int8-b1", "tokens/s"), ("small-int8-trunk-bwd", "positions/s")])
def test_reference_arm_json_line(config, unit):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", config, "--steps", "1",
                          "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0
    assert d["metric"] and d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 1
    assert d["config"]["workload"] == config
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == unit and cb["cores"] >= 1 and cb["kind"] == "port"
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("config", ["small-int8-b32", "small-int8-trunk-bwd"])
def test_reference_arm_runs_on_rank_0_only(config):
    """Under torchrun every rank but 0 exits 0 without work and prints no JSON line."""
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", config, "--gpus", "2",
                          "--steps", "1", "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300,
                         env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
