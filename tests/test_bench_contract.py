"""bench.py's reference arm runs on the host (no GPU) and prints one JSON line with the keys the
contract asks for: the metric and unit of the workload, `impl: reference`, a `cpu_baseline`
describing the run, and an `e2e` object with zero transfer bytes."""
import json
import os
import subprocess
import sys

import numpy as np
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


def test_reference_arm_never_loads_the_product_library():
    """The reference arm builds its weights and ids with the oracle alone (oracle/synth.py), so the
    process that times the reference's CPU path never maps libgpt2q.so."""
    code = ("import runpy, sys; sys.argv = ['bench.py', '--impl', 'reference', '--config', 'small-int8-b1', "
            "'--steps', '1', '--warmup', '1', '--only']; runpy.run_path('bench.py', run_name='__main__'); "
            "maps = open('/proc/self/maps').read(); "
            "print('MAPS', 'libgpt2q' in maps, 'liboracle' in maps)")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "MAPS False True" in out.stdout, out.stdout[-2000:]


def test_both_arms_time_the_same_workload():
    """Same prompts, decode span, staggered offsets and config keys for both arms, at every N."""
    sys.path.insert(0, ROOT)
    import bench

    for name in bench.DECODE:
        wl = bench.WORKLOADS[name]
        for world in (1, 2, 8):
            a, ma = bench.workload_prompts(name, wl, 0, world, 50257, bench.generator(False))
            b, mb = bench.workload_prompts(name, wl, 0, world, 50257, bench.generator(True))
            assert ma == mb and len(a) == len(b) and all(np.array_equal(x, y) for x, y in zip(a, b))
            span = bench.decode_span(wl, 1024, ma)
            plens = [p.size for p in a]
            assert bench.decode_config(name, wl, world, len(a), plens, span) == \
                bench.decode_config(name, wl, world, len(b), [p.size for p in b], span)


@pytest.mark.parametrize("n,span,k", [(1, 64, 20), (32, 128, 20), (256, 256, 20), (32, 128, 127), (5, 10, 1)])
def test_staggered_offsets_cover_the_span(n, span, k):
    sys.path.insert(0, ROOT)
    import bench

    off = bench.stagger(n, span, k)
    assert off.shape == (n,) and off.min() >= 1 and off.max() + k - 1 <= span - 1
    timed = np.concatenate([off + s for s in range(k)])
    assert abs(timed.mean() - span / 2) <= 1.0  # the middle of the decode offsets 0..span-1
    with pytest.raises(ValueError):
        bench.stagger(n, span, span)
