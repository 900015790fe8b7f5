"""Decode throughput of the quantized GPT-2 forward on B200.

    python bench.py [--gpus N --steps K --warmup W] [--config NAME] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

A step is one decode step of a batch of sequences (one new token per sequence).
Default workload (`small-int8-b32`): GPT-2 small, int8 per-group-32 weights
(core.i8.b32.f16scale) from seeded N(0, 0.02) weights, 32 sequences per GPU with
128-token prompts (ids uniform in [0, 50257)), decoding at positions 128..255.
Sequences are independent, so N GPUs each run their own 32 sequences with no
data-path collective (weak scaling).

Printed JSON (rank 0, one line):
  value      decode tokens/s over all ranks with inputs resident in HBM: the timed
             region replays K device-side decode steps (CUDA graph per step, greedy
             argmax feeding the next step), CUDA events on the launch stream,
             max over ranks;
  e2e        the same metric through the public C-ABI call gpt2q_decode with host
             buffers: every step copies its tokens/positions/slots host->device and
             reads the next tokens device->host inside the timed region;
  roofline   the kernel with the largest time share of a decode step: algorithmic bytes
             per launch / steady-state launch time (its launch replayed 20x in a CUDA graph,
             CUDA events on the launch stream), against MEASURED_PEAKS.json hbm_gbs;
  cpu_baseline  the C++ oracle (restatement of the reference CPU forward) timed on
             the host cores on a bounded sample (rank 0, N=1 only).
`--impl reference` times only the reference CPU implementation (the oracle port;
the Rust reference cannot be built here) on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (model, policy, batch, prompt len, decode steps, scaling)
    "small-int8-b32": ("small", "auto", 32, 128, 128, "weak"),      # 32 sequences per GPU, 128 + 128
    "small-int8-b1": ("small", "auto", 1, 64, 64, "weak"),          # single-sequence latency, int8
    "small-int4-b256": ("small", "q4auto", 256, 264, 256, "strong"),  # 256 ragged prompts 16..512, int4
    "medium-int8-prefill": ("medium", "auto", 64, 1024, 1, "strong"),  # 64 x 1024-token prefill
    "xl-int8-tp": ("xl", "auto", 16, 256, 256, "strong"),           # GPT-2 XL, tensor parallel
    "small-int8-trunk-bwd": ("small", "auto", 1, 64, 0, "weak"),    # trunk input gradient of 64 positions
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="small-int8-b32", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-steps", type=int, default=24)
    ap.add_argument("--batch", type=int, default=0, help="override the workload's sequence count (profiling)")
    ap.add_argument("--profile-one-step", action="store_true",
                    help="after the warm-up, run exactly one decode step between cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off) and exit")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def algorithmic_step_bytes(pk, positions, d_local=None) -> float:
    """Bytes one decode step must move: every 2-D weight once, fp32 LN/bias vectors,
    per sequence the K/V rows 0..pos read and row pos written, embed rows."""
    meta = pk.meta
    w = sum(t.data.nbytes for t in pk.tensors.values() if len(t.shape) == 2)
    vec = sum(t.numel * 4 for t in pk.tensors.values() if len(t.shape) == 1)
    d = meta.n_embd
    kv = sum(2.0 * meta.n_layer * d * 4 * (p + 1) + 2.0 * meta.n_layer * d * 4 for p in positions)
    row_bytes = pk.tensors["wte.weight"].data.nbytes / meta.vocab + pk.tensors["wpe.weight"].data.nbytes / meta.n_ctx
    return w + vec + kv + len(positions) * row_bytes


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_pack(model: str, policy: str):
    """Seeded synthetic pack, cached under $TMPDIR so ranks and repeated runs share it."""
    import tempfile

    from smelt_b200 import pack as P
    from smelt_b200 import synth

    meta = P.CONFIGS[model]
    path = os.path.join(tempfile.gettempdir(), f"smelt_b200_pack_{model}_{policy}_seed0.npz")
    lock = path + ".lock"
    for _ in range(3600):
        if os.path.exists(path):
            try:
                z = np.load(path, allow_pickle=False)
                pk = P.Pack(meta)
                for name in z["names"]:
                    shape = tuple(int(v) for v in z[f"shape::{name}"])
                    pk.tensors[str(name)] = P.Tensor(shape, str(z[f"atom::{name}"]), z[f"data::{name}"])
                return pk
            except Exception:
                pass
        try:
            fd = os.open(lock, os.O_CREAT | os.O_EXCL | os.O_WRONLY)
        except FileExistsError:
            time.sleep(1.0)  # another rank is writing the cache
            continue
        try:
            pk = synth.synthetic_pack(meta, policy, seed=0)
            arrays = {"names": np.array(list(pk.tensors))}
            for name, t in pk.tensors.items():
                arrays[f"shape::{name}"] = np.array(t.shape, np.int64)
                arrays[f"atom::{name}"] = np.array(t.atom)
                arrays[f"data::{name}"] = t.data
            tmp = path + f".{os.getpid()}.npz"
            np.savez(tmp, **arrays)
            os.replace(tmp, path)
            return pk
        finally:
            os.close(fd)
            os.unlink(lock)
    raise RuntimeError("timed out waiting for the pack cache")


def prompts_for(rank: int, world: int, n: int, plen: int, vocab: int, ragged: bool):
    """This rank's prompts. Weak scaling (fixed prompts): every rank draws its own n
    prompts. Strong scaling (ragged): the n global prompts are drawn once and split into
    contiguous ranges balanced by token count (smelt_b200.shard)."""
    from smelt_b200 import shard, synth

    if ragged:
        lens = synth.ragged_lengths(n, 16, 512, seed=2)
        ids = synth.prompt_ids(int(lens.sum()), vocab, seed=1)
        offs = np.concatenate([[0], np.cumsum(lens)])
        lo, hi = shard.shard_sequences(lens, world)[rank]
        return [ids[offs[i]:offs[i + 1]] for i in range(lo, hi)]
    lens = np.full(n, plen, np.int32)
    ids = synth.prompt_ids(int(lens.sum()), vocab, seed=1 + 1000 * rank)
    return [ids[i * plen:(i + 1) * plen] for i in range(n)]


def cpu_baseline(pk, plen: int, sample_steps: int, threads: int):
    """Oracle (reference CPU forward restated in C++) on a bounded decode sample."""
    from oracle import oracle as O

    eng = O.Engine(pk.meta.as_dict(), {n: (t.shape, t.atom, t.data) for n, t in pk.tensors.items()}, threads)
    kv = eng.empty_kv()  # attention cost depends on the position, not on cache contents
    eng.step(1, plen, kv)  # warm-up
    t0 = time.perf_counter()
    for s in range(sample_steps):
        eng.step((7 * s + 3) % pk.meta.vocab, plen + 1 + s, kv)
    dt = time.perf_counter() - t0
    return sample_steps / dt, dt


METRICS = {
    "small-int8-b32": "decode tokens/s (GPT-2 small int8)",
    "small-int8-b1": "decode tokens/s (GPT-2 small int8)",
    "small-int4-b256": "decode tokens/s (GPT-2 small int4)",
    "medium-int8-prefill": "prefill tokens/s (GPT-2 medium int8)",
    "xl-int8-tp": "decode tokens/s (GPT-2 XL int8, tensor parallel)",
    "small-int8-trunk-bwd": "trunk input-gradient positions/s (GPT-2 small int8, forward stash + backward)",
}


def bwd_sample(pk, T: int, seed: int = 1):
    """Token ids and the sparse dlogits of the reference's bwparity gate (8 entries per position)."""
    from oracle import backward_oracle as B
    from smelt_b200 import synth

    ids = np.asarray(synth.prompt_ids(T, pk.meta.vocab, seed=seed), np.uint32)
    return ids, B.sparse_dlogits(T, pk.meta.vocab)


def cpu_trunk_baseline(pk, T: int, reps: int):
    """The oracle's trunk backward (f64 numpy, BLAS threads) on T positions, positions/s."""
    from oracle import backward_oracle as B

    W = B.weights64(pk)
    ids, dl = bwd_sample(pk, T)
    dl64 = dl.astype(np.float64)
    _, acts = B.forward_stash(W, pk.meta, ids)  # warm-up
    t0 = time.perf_counter()
    for _ in range(reps):
        _, acts = B.forward_stash(W, pk.meta, ids)
        B.trunk_input_grad(W, pk.meta, acts, dl64)
    dt = time.perf_counter() - t0
    return reps * T / dt, dt


def run_trunk_bwd(args, wl):
    """Trunk input gradient of one 64-position sequence of GPT-2 small int8 (the reference's
    plasticity backward, gpu_backward.rs:651-790): a step is one gpt2q_trunk_input_grad call,
    i.e. the forward with its activation stash plus the backward through the head, ln_f and the
    12 layers, all positions batched. Ranks run independent sequences (weak scaling)."""
    import torch

    from smelt_b200.gpu import Gpu

    model, policy, _batch, T, _dec, scaling = wl
    world, rank, local, dev = dist_setup()
    pk = build_pack(model, policy)
    meta = pk.meta
    ids, dl = bwd_sample(pk, T, seed=1 + rank)
    g = Gpu(pk, device=local, max_seqs=1)
    stream = torch.cuda.Stream(device=dev)
    g.set_stream(stream.cuda_stream)
    for _ in range(max(args.warmup, 3)):
        g.trunk_input_grad(ids, dl)
    # per-kernel times of one call (CUDA events around every launch)
    g.profile(True)
    g.trunk_input_grad(ids, dl)
    prof = g.profile_read()
    g.profile(False)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    l0 = g.launches
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}") as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(args.steps):
            g.trunk_input_grad(ids, dl)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        ms = ev0.elapsed_time(ev1)
    launches = (g.launches - l0) / args.steps
    ms_max = max_over_ranks(ms, world, dev)
    wall_max = max_over_ranks(wall, world, dev)
    hbm, peak_src = peaks()
    top = max(prof.items(), key=lambda kv: kv[1]["ms"])
    kname, kv = top
    per_launch_ms = kv["ms"] / kv["launches"]
    achieved = kv["bytes"] / kv["launches"] / (per_launch_ms / 1e3) / 1e9
    total_ms = sum(v["ms"] for v in prof.values())
    line = {
        "metric": METRICS[args.config], "value": world * T * args.steps / (ms_max / 1e3), "unit": "positions/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "int8xfp32", "data": "synthetic",
        "config": {"workload": args.config, "model": f"gpt2-{model}", "weights": policy, "positions": T,
                   "dlogits": "8 random entries per position (bwparity gate)",
                   "step": "gpt2q_trunk_input_grad: forward stash + backward, host dlogits in, host dx out",
                   "l2": "no flush; the head backward streams the 41 MB int8 wte and 12.9 MB of dlogits"},
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": None, "peak_source": peak_src,
                     "share_of_step": kv["ms"] / total_ms if total_ms else None,
                     "note": "per-launch CUDA events in profiling mode; algorithmic bytes = weights once + dY + dX"},
        "kernels": {k: {"launches": v["launches"], "us_per_launch": 1e3 * v["ms"] / v["launches"]}
                    for k, v in sorted(prof.items(), key=lambda kv: -kv[1]["ms"])[:8]},
        "e2e": {"value": world * T * args.steps / wall_max, "unit": "positions/s",
                "h2d_bytes_per_step": T * meta.vocab * 4 + T * 8, "d2h_bytes_per_step": 2 * T * meta.n_embd * 4,
                "api": "gpt2q_trunk_input_grad"},
        "gpu_launches": int(launches), "clocks": clk.summary(),
    }
    g.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, dt = cpu_trunk_baseline(pk, T, 12)
        line["cpu_baseline"] = {"value": v, "unit": "positions/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"12 calls x {T} positions in {dt:.1f} s: oracle f64 numpy restatement "
                                          "of forward_stash + trunk_input_grad, BLAS threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_reference_trunk(args, wl):
    """The reference arm of the trunk-backward workload: the oracle's restatement on the host
    cores, each step one call on the workload's 64 positions."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    pk = build_pack(wl[0], wl[1])
    cpu_trunk_baseline(pk, wl[3], 1)
    v, dt = cpu_trunk_baseline(pk, wl[3], args.steps)
    line = {
        "impl": "reference", "metric": METRICS[args.config], "value": v, "unit": "positions/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": wl[5], "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": args.config, "model": f"gpt2-{wl[0]}", "weights": wl[1], "positions": wl[3]},
        "cpu_baseline": {"value": v, "unit": "positions/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{args.steps} calls x {wl[3]} positions, oracle f64 numpy restatement"},
        "e2e": {"value": v, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference(args, wl):
    """The reference's CPU path (one token per `Engine::step` call, gpt2.rs:227) on the host cores,
    restated by the oracle, on a bounded sample of this workload: decode workloads time one
    token for each of 2 sequences per step; the prefill workload times 8 consecutive prompt
    tokens per step (the reference prefills by stepping token by token)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    model, policy, batch, plen, dec, _scaling = wl
    pk = build_pack(model, policy)
    threads = os.cpu_count() or 8
    from oracle import oracle as O

    eng = O.Engine(pk.meta.as_dict(), {n: (t.shape, t.atom, t.data) for n, t in pk.tensors.items()}, threads)
    prefill = args.config == "medium-int8-prefill"
    per_step = 8 if prefill else 2
    kvs = [eng.empty_kv() for _ in range(1 if prefill else per_step)]
    from smelt_b200 import synth

    ids = np.asarray(synth.prompt_ids(4096, pk.meta.vocab, seed=1))
    pos = 0
    for w in range(args.warmup):
        if prefill:
            for j in range(per_step):
                eng.step(int(ids[pos % 4096]), pos % pk.meta.n_ctx, kvs[0])
                pos += 1
        else:
            for j in range(per_step):
                eng.step(1, plen + w % dec, kvs[j])
    t0 = time.perf_counter()
    for s in range(args.steps):
        for j in range(per_step):
            if prefill:
                eng.step(int(ids[pos % 4096]), pos % pk.meta.n_ctx, kvs[0])
                pos += 1
            else:
                eng.step((s * 31 + j) % pk.meta.vocab, plen + (args.warmup + s) % dec, kvs[j])
    dt = time.perf_counter() - t0
    tok_s = args.steps * per_step / dt
    sample = (f"{args.steps} steps x {per_step} consecutive prompt tokens of one sequence"
              if prefill else
              f"{args.steps} steps x {per_step} sequences x 1 token at positions {plen}..{plen + dec - 1}")
    line = {
        "impl": "reference", "metric": METRICS[args.config], "value": tok_s, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": wl[5],
        "vs_baseline": None, "dtype": "int8xfp32" if policy == "auto" else "int4xfp32", "data": "synthetic",
        "config": {"workload": args.config, "model": f"gpt2-{model}", "weights": policy, "global_batch": batch,
                   "prompt": plen},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample + f", oracle C++ restatement of gpt2.rs step, "
                                            f"{threads}-thread row split per matmul"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def prefill_flops(meta, T: int) -> float:
    """FLOPs of one prompt of T tokens: 2*T*P_lin + causal attention + last-position head."""
    d, L = meta.n_embd, meta.n_layer
    p_lin = 12 * d * d * L
    return 2.0 * T * p_lin + 2.0 * L * d * T * (T + 1) + 2.0 * d * meta.vocab


def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    return world, rank, local, dev


def max_over_ranks(v: float, world: int, dev) -> float:
    import torch

    t = torch.tensor([v], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def run_prefill(args, wl):
    """GPT-2 medium int8 prefill, 64 prompts of 1024 tokens; a step is their prefill and the greedy token
    after each (generate_greedy with one step), sequences split across ranks (strong
    scaling); tensor-core bound."""
    import torch

    from smelt_b200 import shard, synth
    from smelt_b200.gpu import Gpu

    model, policy, batch, plen, _dec, scaling = wl
    world, rank, local, dev = dist_setup()
    pk = build_pack(model, policy)
    meta = pk.meta
    ids = synth.prompt_ids(batch * plen, meta.vocab, seed=1)
    lo, hi = shard.shard_sequences(np.full(batch, plen), world)[rank]
    prompts = [ids[i * plen:(i + 1) * plen] for i in range(lo, hi)]
    g = Gpu(pk, device=local, max_seqs=max(1, len(prompts)), max_tokens=16384)
    stream = torch.cuda.Stream(device=dev)
    g.set_stream(stream.cuda_stream)

    def step():
        # the prompts fill the context (1024 positions); the single greedy step is the token
        # predicted from the last prompt position, which the prefill already returns
        g.prefill(prompts)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}") as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, world, dev)
    wall_max = max_over_ranks(wall, world, dev)
    tokens = batch * plen * args.steps
    flops_rank = sum(prefill_flops(meta, p.size) for p in prompts)
    peak = 1404.9
    pj = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak_kind = "fallback (sustained)"
    if os.path.exists(pj):
        with open(pj) as f:
            peak = float(json.load(f).get("bf16_tflops_sustained", peak))
        peak_kind = "measured bf16 sustained"
    achieved = flops_rank / (ms / args.steps / 1e3) / 1e12 if prompts else 0.0
    line = {
        "metric": METRICS[args.config], "value": tokens / (ms_max / 1e3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "int8xfp32 (fp16x3 tensor)",
        "data": "synthetic",
        "config": {"workload": args.config, "model": f"gpt2-{model}", "weights": policy, "global_batch": batch,
                   "prompt": plen, "step": "prefill all prompts + greedy token of the last position",
                   "l2": f"inputs larger than L2: {batch * plen * meta.n_embd * 4 / 1e6:.0f} MB of activations per layer"},
        "roofline": {"bound": "tensor", "kernel": "whole prefill step", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                     "flops_per_step_rank": flops_rank,
                     "note": "algorithmic FLOPs (2MNK); the fp16x3 split issues 3x the MMAs"},
        "e2e": {"value": tokens / wall_max, "unit": "tokens/s", "h2d_bytes_per_step": sum(p.size for p in prompts) * 4,
                "d2h_bytes_per_step": len(prompts) * 4, "api": "gpt2q_prefill"},
        "gpu_launches": None, "clocks": clk.summary(),
    }
    g.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_tp(args, wl):
    """GPT-2 XL int8, tensor parallel over the torchrun ranks (NCCL all-reduce
    of the two c_proj partial sums per layer); 16 sequences, decode positions 256..511."""
    import torch

    from smelt_b200 import synth
    from smelt_b200.gpu import Gpu

    model, policy, batch, plen, dec, scaling = wl
    world, rank, local, dev = dist_setup()
    pk = build_pack(model, policy)
    meta = pk.meta
    ids = synth.prompt_ids(batch * plen, meta.vocab, seed=1)
    prompts = [ids[i * plen:(i + 1) * plen] for i in range(batch)]
    if world > 1:
        uid = [torch.cuda.nccl.unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        g = Gpu(pk, device=local, max_seqs=batch, tp_size=world, tp_rank=rank, nccl_id=uid[0])
    else:
        g = Gpu(pk, device=local, max_seqs=batch)
    stream = torch.cuda.Stream(device=dev)
    g.set_stream(stream.cuda_stream)
    g.prefill(prompts)
    span = dec
    done = 0

    def run_steps(k):
        nonlocal done
        while k > 0:
            if done >= span:
                g.prefill(prompts)
                done = 0
            n = min(k, span - done)
            g.decode_steps(n, batch, want_tokens=False)
            done += n
            k -= n

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    l0 = g.launches
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}") as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        k = args.steps
        # prefills that rewind the positions are not decode steps: keep them out of the timing
        timed_ms = 0.0
        while k > 0:
            if done >= span:
                ev1.record(stream)
                torch.cuda.synchronize()
                timed_ms += ev0.elapsed_time(ev1)
                g.prefill(prompts)
                done = 0
                ev0.record(stream)
            n = min(k, span - done)
            g.decode_steps(n, batch, want_tokens=False)
            done += n
            k -= n
        ev1.record(stream)
        torch.cuda.synchronize()
        timed_ms += ev0.elapsed_time(ev1)
    launches = g.launches - l0
    ms_max = max_over_ranks(timed_ms, world, dev)
    weights = sum(t.data.nbytes for t in pk.tensors.values() if len(t.shape) == 2)
    line = {
        "metric": METRICS[args.config], "value": batch * args.steps / (ms_max / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": "int8xfp32", "data": "synthetic",
        "config": {"workload": args.config, "model": f"gpt2-{model}", "weights": policy, "global_batch": batch,
                   "prompt": plen, "parallelism": f"tp{world}" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2: {weights / 1e6:.0f} MB of int8 weights per step"},
        "step_hbm_fraction": None, "gpu_launches": int(launches), "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "whole decode step",
                     "achieved": (weights / world) / (ms_max / args.steps / 1e3) / 1e9, "peak": peaks()[0],
                     "unit": "GB/s", "frac": (weights / world) / (ms_max / args.steps / 1e3) / 1e9 / peaks()[0],
                     "traffic": None, "note": "weight bytes per rank only (KV excluded)"},
        "e2e": None,
    }
    g.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    wl = WORKLOADS[args.config]
    if args.batch > 0:
        wl = (wl[0], wl[1], args.batch) + tuple(wl[3:])
    if args.impl == "reference":
        if args.config == "small-int8-trunk-bwd":
            run_reference_trunk(args, wl)
        else:
            run_reference(args, wl)
        return
    if args.config == "medium-int8-prefill":
        run_prefill(args, wl)
        return
    if args.config == "xl-int8-tp":
        run_tp(args, wl)
        return
    if args.config == "small-int8-trunk-bwd":
        run_trunk_bwd(args, wl)
        return
    import torch

    model, policy, batch, plen, dec, scaling = wl
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from smelt_b200.gpu import Gpu

    pk = build_pack(model, policy)
    meta = pk.meta
    ragged = args.config == "small-int4-b256"
    prompts = prompts_for(rank, world, batch, plen, meta.vocab, ragged)
    n_local = len(prompts)
    max_plen = max(p.size for p in prompts)
    g = Gpu(pk, device=local, max_seqs=n_local, max_tokens=max(8192, max_plen))
    stream = torch.cuda.Stream(device=dev)
    g.set_stream(stream.cuda_stream)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()

    # ---- setup: prefill prompts (untimed), warm-up decode steps ----
    g.prefill(prompts)
    start_pos = np.array([p.size for p in prompts])
    room = int(meta.n_ctx - start_pos.max())
    span = min(dec, room)
    done = 0  # decode steps taken since prefill

    rewind_tok = np.array([p[-1] for p in prompts], np.uint32)
    rewind_slots = np.arange(n_local, dtype=np.int32)

    def run_steps(k):
        # K decode steps cycling over positions start..start+span-1; the step that wraps
        # back to the first decode position is itself a (host-fed) decode step.
        nonlocal done
        while k > 0:
            if done >= span:
                g.decode(rewind_tok, start_pos.astype(np.int32), rewind_slots)
                done = 1
                k -= 1
                continue
            n = min(k, span - done)
            g.decode_steps(n, n_local, want_tokens=False)
            done += n
            k -= n

    run_steps(max(args.warmup, 3))
    barrier()
    if args.profile_one_step:
        torch.cuda.profiler.start()
        run_steps(1)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profiled": "one decode step", "config": args.config, "batch": n_local}))
        return

    # ---- timed region: K device-resident decode steps ----
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    gpu_id = gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}"
    positions_timed = []
    l0 = g.launches
    with ClockSampler(gpu_id) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        # positions each timed step sees (for the roofline bytes)
        d0 = done
        for s in range(args.steps):
            dd = (d0 + s) % span if span else 0
            positions_timed.append(start_pos + dd)
        with torch.cuda.stream(stream):
            ev0.record(stream)
        run_steps(args.steps)
        with torch.cuda.stream(stream):
            ev1.record(stream)
        barrier()
        ms = ev0.elapsed_time(ev1)
        launches = g.launches - l0  # kernels launched inside the timed region
        # keep sampling clocks for at least ~1 s of the same work when the timed region was short
        t_extra = time.perf_counter()
        while time.perf_counter() - t_extra < max(0.0, 1.0 - ms / 1e3):
            run_steps(min(args.steps, 32))
            torch.cuda.synchronize()
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    total_tokens = n_local * args.steps * (world if scaling == "weak" else 1)
    if scaling == "strong":
        total_tokens = batch * args.steps
    value = total_tokens / (ms_max / 1e3)

    # ---- e2e: the public C-ABI call with host buffers, H2D + D2H every step ----
    g.set_stream(None)
    g.prefill(prompts)
    tok = np.ascontiguousarray(g.decode_steps(1, n_local)[0])
    pos = (start_pos + 1).astype(np.int32)
    slots = np.arange(n_local, dtype=np.int32)
    e2e_steps = min(args.steps, room - 1)
    barrier()
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        tok = g.decode(tok, pos + s, slots)
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(e2e_t, op=torch.distributed.ReduceOp.MAX)
    e2e_tokens = n_local * e2e_steps * (world if scaling == "weak" else 1)
    if scaling == "strong":
        e2e_tokens = batch * e2e_steps
    e2e_value = e2e_tokens / float(e2e_t.item())

    # ---- roofline: every kernel type of one decode step timed in steady state (its first
    # launch replayed back to back in a CUDA graph, CUDA events on the launch stream) ----
    g.prefill(prompts)
    persistent = n_local == 1 and g.info()["persistent_decode"]
    if persistent:
        # the whole step is one kernel; a launch runs S consecutive steps
        S = max(1, min(32, span - 1))
        g.decode_steps(S, 1, want_tokens=False)
        g.prefill(prompts)
        pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            pe0.record(stream)
        g.set_stream(stream.cuda_stream)
        g.decode_steps(S, 1, want_tokens=False)
        with torch.cuda.stream(stream):
            pe1.record(stream)
        torch.cuda.synchronize()
        g.set_stream(None)
        pos_s = [start_pos + k for k in range(S)]
        kt = {"k_decode_persistent": {"us": pe0.elapsed_time(pe1) * 1e3, "per_step": 1.0 / S,
                                      "bytes": sum(algorithmic_step_bytes(pk, p) for p in pos_s)}}
    else:
        kt = g.profile_kernels(reps=20)
    name, rec = max(kt.items(), key=lambda kv: kv[1]["us"] * kv[1]["per_step"])
    per_launch_bytes = rec["bytes"]
    per_launch_ms = rec["us"] / 1e3
    hbm, peak_kind = peaks()
    achieved = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tfile):
        with open(tfile) as f:
            tj = json.load(f)
        traffic = tj.get(args.config, {}).get(name)
        if persistent and tj.get(args.config, {}).get("k_decode_persistent_per_step"):
            traffic = tj[args.config]["k_decode_persistent_per_step"] * round(1 / rec["per_step"])
    step_bytes = statistics.mean(algorithmic_step_bytes(pk, p) for p in positions_timed)

    line = {
        "metric": METRICS[args.config],
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": "int8xfp32" if policy == "auto" else "int4xfp32", "data": "synthetic",
        "config": {"workload": args.config, "model": f"gpt2-{model}", "weights": policy,
                   "batch_per_gpu": n_local, "global_batch": n_local * world if scaling == "weak" else batch,
                   "prompt": plen, "decode_positions": f"{int(start_pos.min())}..{int(start_pos.max()) + span - 1}",
                   "kv_dtype": "fp32", "parallelism": f"sequence-sharded x{world}",
                   "l2": f"inputs larger than L2: {step_bytes / 1e6:.0f} MB moved per step vs 126 MB L2"},
        "step_hbm_fraction": (step_bytes / (ms_max / args.steps / 1e3) / 1e9) / hbm,
        "roofline": {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic, "peak_source": peak_kind,
                     "bytes_per_launch": per_launch_bytes, "us_per_launch": rec["us"],
                     "timing": ("one launch of %d consecutive steps, CUDA events" % round(1 / rec["per_step"]))
                     if persistent else "graph of 20 back-to-back launches of the step's own launch, CUDA events"},
        "kernels": {k: {"us_per_launch": round(v["us"], 3), "per_step": v["per_step"],
                        "step_share": round(v["us"] * v["per_step"] / (ms_max / args.steps * 1e3), 4)}
                    for k, v in kt.items()},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": n_local * 12,
                "d2h_bytes_per_step": n_local * 4, "api": "gpt2q_decode (host tok/pos/slot in, next tokens out)"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = min(8, os.cpu_count() or 8)
        tok_s, dt = cpu_baseline(pk, plen, args.cpu_sample_steps, threads)
        line["cpu_baseline"] = {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"{args.cpu_sample_steps} single-sequence decode steps at positions "
                                          f"{plen + 1}..{plen + args.cpu_sample_steps} ({dt:.1f} s), oracle C++ "
                                          f"restatement of the reference step, {threads}-thread row split per matmul"}
    g.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
