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


@pytest.mark.parametrize("config,unit", [("small-int8-b1", "tokens/s"), ("small-int8-trunk-bwd", "positions/s"),
                                         ("medium-int8-prefill", "tokens/s")])
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


@pytest.mark.parametrize("n,span,steps", [(1, 64, 100), (1, 64, 20), (32, 128, 100), (256, 256, 100), (5, 10, 23)])
def test_every_timed_chunk_starts_inside_the_fill(n, span, steps):
    """The timed region runs `steps` decode steps in chunks of at most span - 1, each from a
    rewind to staggered offsets; a shorter last chunk staggers further in. Every rewind feeds
    the token decoded at offset o - 1, which the untimed fill must hold."""
    sys.path.insert(0, ROOT)
    import bench

    k1 = min(steps, span - 1)
    chunks = [k1] * (steps // k1) + ([steps % k1] if steps % k1 else [])
    fill = max(span - 2, 3)  # as measure_decode
    for k in chunks:
        off = bench.stagger(n, span, k)
        assert 1 <= off.min() and off.max() - 1 <= fill and off.max() + k - 1 <= span - 1
