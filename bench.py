"""Decode throughput of the quantized GPT-2 forward on B200.

    python bench.py [--gpus N --steps K --warmup W] [--config NAME] [--impl ours|reference] [--only]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

A step is one decode step of a batch of sequences (one new token per sequence).
Default workload (`small-int8-b32`): GPT-2 small, int8 per-group-32 weights
(core.i8.b32.f16scale) from seeded N(0, 0.02) weights, 32 sequences per GPU with
128-token prompts (ids uniform in [0, 50257)), decoding positions 128..255.
Sequences are independent, so N GPUs each run their own 32 sequences with no
data-path collective (weak scaling). The default run also reports, in
`workloads`, the single-sequence decode (`small-int8-b1`, prompt 64, decode 64)
and the int4 decode of 256 ragged prompts of 16..512 tokens (`small-int4-b256`,
decode 256, sequences split across the ranks), and the GPT-2 medium int8 prefill of
64 prompts of 1024 tokens (`medium-int8-prefill`, min(K, 5) timed prefill steps,
prompts split across the ranks); `--only` skips them. With N >= 2 it adds
`xl-int8-tp`, GPT-2 XL tensor parallel over the N ranks.

Timed decode steps are spread over each workload's whole decode span: before the
timed region every sequence is rewound to its own start offset o_i (spread over
1..span-K), so sequence i runs its K timed steps at positions prompt_i + o_i ..
prompt_i + o_i + K - 1 and the mean position is the middle of the span.

Printed JSON (rank 0, one line), for the headline and each sub-workload:
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
  cpu_baseline  the C++ oracle (restatement of the reference CPU forward, 8-thread row
             split per matmul as the reference) timed on the host cores at positions
             sampled from the timed steps (rank 0, N=1 only).
`--impl reference` times only the reference CPU implementation (the oracle port; the
Rust reference cannot be built here) on the same workloads, with weights and token ids
made by the oracle alone (oracle/synth.py), so that process never loads the product
library.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from types import SimpleNamespace

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
DECODE = ("small-int8-b32", "small-int8-b1", "small-int4-b256")
SUB_WORKLOADS = ("small-int8-b1", "small-int4-b256")  # reported inside the default run's line
RAGGED = (16, 512)  # prompt lengths of small-int4-b256
REF_THREADS = 8  # gpt2.rs:154: matmul splits the rows over min(8, rows) scoped threads
TP_PARITY_PROMPT, TP_PARITY_STEPS = 16, 8

METRICS = {
    "small-int8-b32": "decode tokens/s (GPT-2 small int8)",
    "small-int8-b1": "decode tokens/s (GPT-2 small int8)",
    "small-int4-b256": "decode tokens/s (GPT-2 small int4)",
    "medium-int8-prefill": "prefill tokens/s (GPT-2 medium int8)",
    "xl-int8-tp": "decode tokens/s (GPT-2 XL int8, tensor parallel)",
    "small-int8-trunk-bwd": "trunk input-gradient positions/s (GPT-2 small int8, forward stash + backward)",
}
L2_NOTE = "no flush: inputs larger than L2 (every step reads all weights and every sequence's K/V, > 126 MB)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="small-int8-b32", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--only", action="store_true", help="report the selected workload alone (no sub-workloads)")
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


def bf16_sustained():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f).get("bf16_tflops_sustained", 1404.9)), "measured bf16 sustained"
    return 1404.9, "fallback (sustained)"


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

    def __init__(self, dev):
        import torch

        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        self.gpu_id = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
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


def _cached_npz(path: str, make):
    """Load name -> (shape, atom, bytes) from `path`, or make it once (ranks share the file)."""
    lock = path + ".lock"
    for _ in range(3600):
        if os.path.exists(path):
            try:
                z = np.load(path, allow_pickle=False)
                return {str(n): (tuple(int(v) for v in z[f"shape::{n}"]), str(z[f"atom::{n}"]), z[f"data::{n}"])
                        for n in z["names"]}
            except Exception:
                pass
        try:
            fd = os.open(lock, os.O_CREAT | os.O_EXCL | os.O_WRONLY)
        except FileExistsError:
            time.sleep(1.0)  # another rank is writing the cache
            continue
        try:
            tensors = make()
            arrays = {"names": np.array(list(tensors))}
            for name, (shape, atom, data) in tensors.items():
                arrays[f"shape::{name}"] = np.array(shape, np.int64)
                arrays[f"atom::{name}"] = np.array(atom)
                arrays[f"data::{name}"] = data
            tmp = path + f".{os.getpid()}.npz"
            np.savez(tmp, **arrays)
            os.replace(tmp, path)
            return tensors
        finally:
            os.close(fd)
            os.unlink(lock)
    raise RuntimeError("timed out waiting for the weight cache")


def build_pack(model: str, policy: str):
    """Seeded synthetic pack (the product's generator), cached under $TMPDIR."""
    import tempfile

    from smelt_b200 import pack as P
    from smelt_b200 import synth

    meta = P.CONFIGS[model]

    def make():
        pk = synth.synthetic_pack(meta, policy, seed=0)
        return {n: (t.shape, t.atom, t.data) for n, t in pk.tensors.items()}

    tensors = _cached_npz(os.path.join(tempfile.gettempdir(), f"smelt_b200_pack_{model}_{policy}_seed0.npz"), make)
    pk = P.Pack(meta)
    for name, (shape, atom, data) in tensors.items():
        pk.tensors[name] = P.Tensor(shape, atom, data)
    return pk


def oracle_model(model: str, policy: str):
    """(meta dict, tensors) of the same seeded model made by the oracle alone (oracle/synth.py);
    the reference arm uses this so that it never loads the product library."""
    import tempfile

    from oracle import synth as OS

    meta = OS.MODELS[model]
    path = os.path.join(tempfile.gettempdir(), f"smelt_oracle_model_{model}_{policy}_seed0.npz")
    return meta, _cached_npz(path, lambda: OS.synthetic_tensors(meta, policy, seed=0))


def generator(oracle_side: bool):
    """Token-id / prompt-length generator: the product's or the oracle's (identical values)."""
    if oracle_side:
        from oracle import synth as gen
    else:
        from smelt_b200 import synth as gen
    return gen


# ------------------------------------------------------------------ decode workloads
def workload_prompts(name: str, wl, rank: int, world: int, vocab: int, gen):
    """This rank's prompts. Weak scaling (fixed prompts): every rank draws its own n
    prompts. Strong scaling (ragged): the n global prompts are drawn once and split into
    contiguous ranges balanced by token count (smelt_b200.shard). Also returns the longest
    prompt of the whole job (it bounds the decode span)."""
    from smelt_b200 import shard  # pure-Python partitioning (no native code)

    _model, _policy, n, plen, _dec, _scaling = wl
    if name == "small-int4-b256":
        lens = gen.ragged_lengths(n, RAGGED[0], RAGGED[1], seed=2)
        ids = gen.prompt_ids(int(lens.sum()), vocab, seed=1)
        offs = np.concatenate([[0], np.cumsum(lens)])
        lo, hi = shard.shard_sequences(lens, world)[rank]
        return [ids[offs[i]:offs[i + 1]] for i in range(lo, hi)], int(lens.max())
    ids = gen.prompt_ids(n * plen, vocab, seed=1 + 1000 * rank)
    return [ids[i * plen:(i + 1) * plen] for i in range(n)], plen


def decode_span(wl, n_ctx: int, max_plen: int) -> int:
    return min(wl[4], n_ctx - max_plen)


def stagger(n: int, span: int, k: int) -> np.ndarray:
    """Start offsets o_i in [1, span - k] of n sequences that each run k timed steps at
    offsets o_i .. o_i + k - 1 past their prompt: spread evenly, so the timed positions cover
    the decode span and their mean is its middle."""
    hi = span - k
    if hi < 1:
        raise ValueError(f"{k} steps do not fit a decode span of {span}")
    if n == 1:
        return np.array([1 + (hi - 1) // 2])
    return 1 + np.round(np.arange(n) * (hi - 1) / (n - 1)).astype(np.int64)


def decode_config(name: str, wl, world: int, n_local: int, plens, span: int) -> dict:
    model, policy, batch, plen, _dec, scaling = wl
    return {"workload": name, "model": f"gpt2-{model}", "weights": policy, "batch_per_gpu": n_local,
            "global_batch": batch * world if scaling == "weak" else batch,
            "prompt": f"{RAGGED[0]}..{RAGGED[1]} ragged" if name == "small-int4-b256" else plen,
            "decode_positions": f"{int(min(plens))}..{int(max(plens)) + span - 1}",
            "timed_positions": "staggered: sequence i runs its timed steps from prompt_i + o_i, "
                               "o_i spread evenly over 1..span-steps",
            "kv_dtype": "fp32", "parallelism": f"sequence-sharded x{world}", "l2": L2_NOTE}


class DecodeRun:
    """A handle holding prefilled sequences whose greedy continuation is known, so that any
    sequence can be rewound to any decode offset with its own next token."""

    def __init__(self, g, prompts, span: int, fill: int):
        self.g = g
        self.n = len(prompts)
        self.plen = np.array([p.size for p in prompts], np.int64)
        self.span = span
        self.slots = np.arange(self.n, dtype=np.int32)
        self.first = g.prefill(prompts)  # the token fed at offset 0 (position prompt_i)
        # untimed greedy decode: fills the K/V rows every rewind reads (and warms up)
        self.fill = g.decode_steps(fill, self.n) if fill > 0 else np.zeros((0, self.n), np.uint32)

    def token_fed_at(self, off: np.ndarray) -> np.ndarray:
        return np.array([self.first[i] if o == 0 else self.fill[o - 1][i] for i, o in enumerate(off)], np.uint32)

    def rewind(self, k: int) -> tuple:
        """One host-fed decode step per sequence at offset o_i - 1 (untimed), leaving every
        sequence ready to decode at offset o_i; returns (offsets, next tokens)."""
        off = stagger(self.n, self.span, k)
        nxt = self.g.decode(self.token_fed_at(off - 1), (self.plen + off - 1).astype(np.int32), self.slots)
        return off, nxt

    def positions(self, off, k: int):
        return [self.plen + off + s for s in range(k)]


def cpu_decode_rate(eng, positions, vocab: int) -> tuple:
    """The oracle's Engine::step at the given positions (attention cost depends on the position,
    not on the cache contents): tokens/s and seconds."""
    kv = eng.empty_kv()
    eng.step(1, int(positions[0]), kv)  # warm-up
    t0 = time.perf_counter()
    for j, p in enumerate(positions):
        eng.step((7 * j + 3) % vocab, int(p), kv)
    dt = time.perf_counter() - t0
    return len(positions) / dt, dt


def sample_positions(positions, count: int) -> np.ndarray:
    allp = np.sort(np.concatenate([np.asarray(p).ravel() for p in positions]))
    return allp[np.linspace(0, allp.size - 1, count).round().astype(int)]


def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not torch.distributed.is_initialized():
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    return world, rank, local, dev


def max_over_ranks(v: float, world: int, dev) -> float:
    import torch

    t = torch.tensor([v], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()


def measure_decode(args, name: str, wl, world: int, rank: int, local: int, dev) -> dict | None:
    """One decode workload on this rank's GPU; returns the rank-0 JSON record."""
    import torch

    from smelt_b200.gpu import Gpu

    model, policy, batch, plen, dec, scaling = wl
    pk = build_pack(model, policy)
    meta = pk.meta
    prompts, max_plen = workload_prompts(name, wl, rank, world, meta.vocab, generator(False))
    n_local = len(prompts)
    span = decode_span(wl, meta.n_ctx, max_plen)
    K = args.steps
    k1 = min(K, span - 1)  # steps per timed chunk (a chunk never leaves the span)
    g = Gpu(pk, device=local, max_seqs=n_local, max_tokens=max(8192, max(p.size for p in prompts)))
    stream = torch.cuda.Stream(device=dev)
    g.set_stream(stream.cuda_stream)
    # every chunk of the timed region starts from offsets <= span - 1 (a shorter last chunk
    # staggers further in), so the fill decodes the whole span up to that
    fill = max(span - 2, max(args.warmup, 3))
    run = DecodeRun(g, prompts, span, fill)
    barrier(world)
    if args.profile_one_step:
        run.rewind(k1)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        g.decode_steps(1, n_local, want_tokens=False)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        g.close()
        return {"profiled": "one decode step", "config": name, "batch": n_local}

    # ---- timed region: K device-resident decode steps, in chunks that each start from a rewind ----
    positions_timed, ms, launches = [], 0.0, 0
    with ClockSampler(dev) as clk:
        left = K
        while left > 0:
            k = min(left, k1)
            off, _ = run.rewind(k)
            barrier(world)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0 = g.launches
            ev0.record(stream)
            g.decode_steps(k, n_local, want_tokens=False)
            ev1.record(stream)
            torch.cuda.synchronize()
            ms += ev0.elapsed_time(ev1)
            launches += g.launches - l0  # kernels launched inside the timed region
            positions_timed += run.positions(off, k)
            left -= k
        # keep sampling clocks for at least ~1 s of the same work when the timed region was short
        t_extra = time.perf_counter()
        while time.perf_counter() - t_extra < max(0.0, 1.0 - ms / 1e3):
            run.rewind(k1)
            g.decode_steps(k1, n_local, want_tokens=False)
            torch.cuda.synchronize()
    ms_max = max_over_ranks(ms, world, dev)
    total_tokens = (n_local * world if scaling == "weak" else batch) * K
    value = total_tokens / (ms_max / 1e3)

    # ---- e2e: the public C-ABI call with host buffers, H2D + D2H every step, same positions ----
    off, tok = run.rewind(k1)
    pos0 = (run.plen + off).astype(np.int32)
    barrier(world)
    t0 = time.perf_counter()
    for s in range(k1):
        tok = g.decode(tok, pos0 + s, run.slots)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, dev)
    e2e_value = (n_local * world if scaling == "weak" else batch) * k1 / e2e_s

    # ---- roofline: the dominant kernel of a decode step at the staggered positions ----
    persistent = n_local == 1 and g.info()["persistent_decode"]
    if persistent:
        # the whole step is one kernel; one launch runs S consecutive steps
        S = min(32, k1)
        off, _ = run.rewind(S)
        pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pe0.record(stream)
        g.decode_steps(S, 1, want_tokens=False)
        pe1.record(stream)
        torch.cuda.synchronize()
        kt = {"k_decode_persistent": {"us": pe0.elapsed_time(pe1) * 1e3, "per_step": 1.0 / S,
                                      "bytes": sum(algorithmic_step_bytes(pk, p) for p in run.positions(off, S))}}
    else:
        run.rewind(k1)
        kt = g.profile_kernels(reps=20)
    kname, rec = max(kt.items(), key=lambda kv: kv[1]["us"] * kv[1]["per_step"])
    hbm, peak_kind = peaks()
    achieved = rec["bytes"] / (rec["us"] / 1e6) / 1e9
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tfile):
        with open(tfile) as f:
            tj = json.load(f).get(name, {})
        traffic = tj.get(kname)
        if persistent and tj.get("k_decode_persistent_per_step"):
            traffic = tj["k_decode_persistent_per_step"] * round(1 / rec["per_step"])
    step_bytes = statistics.mean(algorithmic_step_bytes(pk, p) for p in positions_timed)
    line = {
        "metric": METRICS[name], "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "int8xfp32" if policy == "auto" else "int4xfp32", "data": "synthetic",
        "config": decode_config(name, wl, world, n_local, run.plen, span),
        "step_bytes": step_bytes,
        "step_hbm_fraction": (step_bytes / (ms_max / K / 1e3) / 1e9) / hbm,
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic, "peak_source": peak_kind,
                     "bytes_per_launch": rec["bytes"], "us_per_launch": rec["us"],
                     "timing": ("one launch of %d consecutive steps, CUDA events" % round(1 / rec["per_step"]))
                     if persistent else "graph of 20 back-to-back launches of the step's own launch, CUDA events"},
        "kernels": {k: {"us_per_launch": round(v["us"], 3), "per_step": v["per_step"],
                        "step_share": round(v["us"] * v["per_step"] / (ms_max / K * 1e3), 4)}
                    for k, v in kt.items()},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "steps": k1, "h2d_bytes_per_step": n_local * 12,
                "d2h_bytes_per_step": n_local * 4, "api": "gpt2q_decode (host tok/pos/slot in, next tokens out)"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    g.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O

        eng = O.Engine(meta.as_dict(), {n: (t.shape, t.atom, t.data) for n, t in pk.tensors.items()}, REF_THREADS)
        sample = sample_positions(positions_timed, args.cpu_sample_steps)
        tok_s, dt = cpu_decode_rate(eng, sample, meta.vocab)
        line["cpu_baseline"] = {
            "value": tok_s, "unit": "tokens/s", "cores": REF_THREADS, "kind": "port",
            "sample": f"{sample.size} single-sequence decode steps at positions {int(sample.min())}..{int(sample.max())} "
                      f"sampled evenly from the timed steps ({dt:.1f} s), oracle C++ restatement of the "
                      f"reference step, {REF_THREADS}-thread row split per matmul"}
    return line


def run_decode(args, wl):
    world, rank, local, dev = dist_setup()
    line = measure_decode(args, args.config, wl, world, rank, local, dev)
    if not args.only and args.config == "small-int8-b32" and not args.profile_one_step and args.batch == 0:
        line["workloads"] = {}
        for name in SUB_WORKLOADS:
            line["workloads"][name] = measure_decode(args, name, WORKLOADS[name], world, rank, local, dev)
        pname = "medium-int8-prefill"
        line["workloads"][pname] = measure_prefill(args, pname, WORKLOADS[pname], world, rank, local, dev,
                                                   steps=min(args.steps, PREFILL_SUB_STEPS))
        if world > 1:
            line["workloads"]["xl-int8-tp"] = measure_tp(args, WORKLOADS["xl-int8-tp"], world, rank, local, dev,
                                                         parity=True)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch

        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------ reference arm
def oracle_engine(model: str, policy: str):
    from oracle import oracle as O

    meta, tensors = oracle_model(model, policy)
    return meta, O.Engine(meta, tensors, REF_THREADS)


def reference_decode(args, name: str, wl, world: int) -> dict:
    """The reference's CPU path (one token per Engine::step call, gpt2.rs:227) on the host
    cores, restated by the oracle, at the positions our arm times: step s runs one token of
    `per_step` sequences, each at the position its own timed step s has."""
    model, policy, batch, plen, dec, scaling = wl
    meta, eng = oracle_engine(model, policy)
    prompts, max_plen = workload_prompts(name, wl, 0, world, meta["vocab"], generator(True))
    n_local = len(prompts)
    span = decode_span(wl, meta["n_ctx"], max_plen)
    k1 = min(args.steps, span - 1)
    plens = np.array([p.size for p in prompts], np.int64)
    off = stagger(n_local, span, k1)
    per_step = min(2, n_local)
    kv = eng.empty_kv()

    def one(s: int):
        for j in range(per_step):
            i = (s * per_step + j) % n_local
            eng.step((s * 31 + j) % meta["vocab"], int(plens[i] + off[i] + s % k1), kv)

    for w in range(args.warmup):
        one(w)
    t0 = time.perf_counter()
    for s in range(args.steps):
        one(s)
    dt = time.perf_counter() - t0
    tok_s = args.steps * per_step / dt
    return {
        "impl": "reference", "metric": METRICS[name], "value": tok_s, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "int8xfp32" if policy == "auto" else "int4xfp32",
        "data": "synthetic", "config": decode_config(name, wl, world, n_local, plens, span),
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": REF_THREADS, "kind": "port",
                         "sample": f"{args.steps} steps x {per_step} sequences x 1 token at each sequence's timed "
                                   f"positions, oracle C++ restatement of gpt2.rs step (weights and ids from the "
                                   f"oracle), {REF_THREADS}-thread row split per matmul"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_prefill(args, name: str, wl, world: int, steps: int | None = None) -> dict:
    """Prefill as the reference does it, one Engine::step per prompt token (gpt2.rs:373-381):
    each step times 8 consecutive prompt tokens of one sequence."""
    model, policy, batch, plen, _dec, scaling = wl
    meta, eng = oracle_engine(model, policy)
    ids = generator(True).prompt_ids(batch * plen, meta["vocab"], seed=1)
    kv = eng.empty_kv()
    per_step, pos = 8, 0
    steps = args.steps if steps is None else steps
    warmup = min(args.warmup, steps)

    def one():
        nonlocal pos
        for _ in range(per_step):
            eng.step(int(ids[pos % ids.size]), pos % plen, kv)
            pos += 1

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = time.perf_counter() - t0
    tok_s = steps * per_step / dt
    return {
        "impl": "reference", "metric": METRICS[name], "value": tok_s, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": dt * 1e3 / steps, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "int8xfp32", "data": "synthetic",
        "config": prefill_config(name, wl, world),
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": REF_THREADS, "kind": "port",
                         "sample": f"{steps} steps x {per_step} consecutive prompt tokens of one sequence, "
                                   f"oracle C++ restatement of gpt2.rs step, {REF_THREADS}-thread row split"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_tp(args, wl, world: int) -> dict:
    """GPT-2 XL decode as the reference does it (one Engine::step per token, single process)."""
    model, policy, batch, plen, dec, scaling = wl
    meta, eng = oracle_engine(model, policy)
    kv = eng.empty_kv()
    k1 = min(args.steps, dec - 1)

    def one(s: int):
        eng.step((s * 31) % meta["vocab"], plen + (s % k1), kv)

    for w in range(args.warmup):
        one(w)
    t0 = time.perf_counter()
    for s in range(args.steps):
        one(s)
    dt = time.perf_counter() - t0
    tok_s = args.steps / dt
    return {
        "impl": "reference", "metric": METRICS["xl-int8-tp"], "value": tok_s, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "int8xfp32", "data": "synthetic",
        "config": tp_config(wl, world),
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": REF_THREADS, "kind": "port",
                         "sample": f"{args.steps} single-token steps at positions {plen}..{plen + k1 - 1}, oracle C++ "
                                   f"restatement of gpt2.rs step, {REF_THREADS}-thread row split"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference(args, wl):
    """`--impl reference`: rank 0 alone times the oracle's restatement of the reference's CPU
    path on the host cores and prints the line; other ranks exit without work."""
    world = int(os.environ.get("WORLD_SIZE", str(max(1, args.gpus))))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.config == "small-int8-trunk-bwd":
        line = reference_trunk(args, wl, world)
    elif args.config == "medium-int8-prefill":
        line = reference_prefill(args, args.config, wl, world)
    elif args.config == "xl-int8-tp":
        line = reference_tp(args, wl, world)
    else:
        line = reference_decode(args, args.config, wl, world)
        if not args.only and args.config == "small-int8-b32" and args.batch == 0:
            line["workloads"] = {n: reference_decode(args, n, WORKLOADS[n], world) for n in SUB_WORKLOADS}
            pname = "medium-int8-prefill"
            line["workloads"][pname] = reference_prefill(args, pname, WORKLOADS[pname], world,
                                                         steps=min(args.steps, PREFILL_SUB_STEPS))
            if world > 1:
                line["workloads"]["xl-int8-tp"] = reference_tp(args, WORKLOADS["xl-int8-tp"], world)
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ trunk backward
def bwd_sample(vocab: int, T: int, gen, seed: int = 1):
    """Token ids and the sparse dlogits of the reference's bwparity gate (8 entries per position)."""
    from oracle import backward_oracle as B

    ids = np.asarray(gen.prompt_ids(T, vocab, seed=seed), np.uint32)
    return ids, B.sparse_dlogits(T, vocab)


def cpu_trunk_rate(W: dict, meta, ids, dl, reps: int) -> tuple:
    """The oracle's trunk backward (f64 numpy, BLAS threads): positions/s and seconds."""
    from oracle import backward_oracle as B

    dl64 = dl.astype(np.float64)
    B.forward_stash(W, meta, ids)  # warm-up
    t0 = time.perf_counter()
    for _ in range(reps):
        _, acts = B.forward_stash(W, meta, ids)
        B.trunk_input_grad(W, meta, acts, dl64)
    dt = time.perf_counter() - t0
    return reps * ids.size / dt, dt


def run_trunk_bwd(args, wl):
    """Trunk input gradient of one 64-position sequence of GPT-2 small int8 (the reference's
    plasticity backward, gpu_backward.rs:651-790): a step is one gpt2q_trunk_input_grad call,
    i.e. the forward with its activation stash plus the backward through the head, ln_f and the
    12 layers, all positions batched. Ranks run independent sequences (weak scaling)."""
    import torch

    from oracle import backward_oracle as B
    from smelt_b200.gpu import Gpu

    model, policy, _batch, T, _dec, scaling = wl
    world, rank, local, dev = dist_setup()
    pk = build_pack(model, policy)
    meta = pk.meta
    ids, dl = bwd_sample(meta.vocab, T, generator(False), seed=1 + rank)
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
    barrier(world)
    l0 = g.launches
    with ClockSampler(dev) as clk:
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
    kname, kv = max(prof.items(), key=lambda kv: kv[1]["ms"])
    per_launch_ms = kv["ms"] / kv["launches"]
    achieved = kv["bytes"] / kv["launches"] / (per_launch_ms / 1e3) / 1e9
    total_ms = sum(v["ms"] for v in prof.values())
    line = {
        "metric": METRICS[args.config], "value": world * T * args.steps / (ms_max / 1e3), "unit": "positions/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "int8xfp32", "data": "synthetic",
        "config": trunk_config(wl),
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
        W = B.weights64(pk)
        v, dt = cpu_trunk_rate(W, meta, ids, dl, 12)
        line["cpu_baseline"] = {"value": v, "unit": "positions/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"12 calls x {T} positions in {dt:.1f} s: oracle f64 numpy restatement "
                                          "of forward_stash + trunk_input_grad, BLAS threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def trunk_config(wl) -> dict:
    model, policy, _b, T, _d, _s = wl
    return {"workload": "small-int8-trunk-bwd", "model": f"gpt2-{model}", "weights": policy, "positions": T,
            "dlogits": "8 random entries per position (bwparity gate)",
            "step": "gpt2q_trunk_input_grad: forward stash + backward, host dlogits in, host dx out",
            "l2": "no flush; the head backward streams the 41 MB int8 wte and 12.9 MB of dlogits"}


def reference_trunk(args, wl, world: int) -> dict:
    """The reference arm of the trunk-backward workload: the oracle's restatement on the host
    cores (weights dequantised by the oracle), each step one call on the workload's 64 positions."""
    model, policy, _b, T, _d, scaling = wl
    meta, eng = oracle_engine(model, policy)
    W = {n: eng.vec_f32(n).reshape(eng.shapes[n]).astype(np.float64) for n in eng.shapes}
    m = SimpleNamespace(**meta)
    ids, dl = bwd_sample(meta["vocab"], T, generator(True))
    cpu_trunk_rate(W, m, ids, dl, 1)
    v, dt = cpu_trunk_rate(W, m, ids, dl, args.steps)
    return {
        "impl": "reference", "metric": METRICS[args.config], "value": v, "unit": "positions/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": trunk_config(wl),
        "cpu_baseline": {"value": v, "unit": "positions/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{args.steps} calls x {T} positions, oracle f64 numpy restatement"},
        "e2e": {"value": v, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------ prefill
def prefill_flops(n_embd: int, n_layer: int, vocab: int, T: int) -> float:
    """FLOPs of one prompt of T tokens: 2*T*P_lin + causal attention + last-position head."""
    p_lin = 12 * n_embd * n_embd * n_layer
    return 2.0 * T * p_lin + 2.0 * n_layer * n_embd * T * (T + 1) + 2.0 * n_embd * vocab


def prefill_config(name: str, wl, world: int) -> dict:
    model, policy, batch, plen, _dec, _s = wl
    return {"workload": name, "model": f"gpt2-{model}", "weights": policy, "global_batch": batch, "prompt": plen,
            "parallelism": f"sequence-sharded x{world}", "step": "prefill all prompts + greedy token of the last position",
            "l2": f"no flush: inputs larger than L2 ({batch * plen * 1024 * 4 / 1e6:.0f} MB of activations per layer)"}


PREFILL_SUB_STEPS = 5  # timed prefill steps (64 x 1024 tokens each) of the sub-result in the default line


def measure_prefill(args, name: str, wl, world: int, rank: int, local: int, dev, steps: int | None = None) -> dict:
    """GPT-2 medium int8 prefill, 64 prompts of 1024 tokens; a step is their prefill and the greedy
    token after each (generate_greedy with one step), sequences split across ranks (strong
    scaling); tensor-core bound. Returns the rank-0 record."""
    import torch

    from smelt_b200 import shard, synth
    from smelt_b200.gpu import Gpu

    model, policy, batch, plen, _dec, scaling = wl
    steps = args.steps if steps is None else steps
    pk = build_pack(model, policy)
    meta = pk.meta
    ids = synth.prompt_ids(batch * plen, meta.vocab, seed=1)
    lo, hi = shard.shard_sequences(np.full(batch, plen), world)[rank]
    prompts = [ids[i * plen:(i + 1) * plen] for i in range(lo, hi)]
    g = Gpu(pk, device=local, max_seqs=max(1, len(prompts)), max_tokens=16384)
    stream = torch.cuda.Stream(device=dev)
    g.set_stream(stream.cuda_stream)
    warmup = max(args.warmup, 3) if steps == args.steps else 3
    for _ in range(warmup):
        g.prefill(prompts)
    barrier(world)
    with ClockSampler(dev) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = g.launches
        t0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(steps):
            # the single greedy step is the token predicted from the last prompt position,
            # which the prefill returns
            g.prefill(prompts)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        ms = ev0.elapsed_time(ev1)
        launches = g.launches - l0
    ms_max = max_over_ranks(ms, world, dev)
    wall_max = max_over_ranks(wall, world, dev)
    tokens = batch * plen * steps
    flops_rank = sum(prefill_flops(meta.n_embd, meta.n_layer, meta.vocab, p.size) for p in prompts)
    peak, peak_kind = bf16_sustained()
    achieved = flops_rank / (ms / steps / 1e3) / 1e12 if prompts else 0.0
    line = {
        "metric": METRICS[name], "value": tokens / (ms_max / 1e3), "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms_max / steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "int8xfp32 (fp16 split tensor)",
        "data": "synthetic", "config": prefill_config(name, wl, world),
        "roofline": {"bound": "tensor", "kernel": "whole prefill step", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None, "peak_source": peak_kind,
                     "flops_per_step_rank": flops_rank,
                     "note": "algorithmic FLOPs (2MNK); the fp16 hi/lo split issues more MMAs than that"},
        "e2e": {"value": tokens / wall_max, "unit": "tokens/s", "h2d_bytes_per_step": sum(p.size for p in prompts) * 4,
                "d2h_bytes_per_step": len(prompts) * 4, "api": "gpt2q_prefill"},
        "gpu_launches": int(launches), "clocks": clk.summary(),
    }
    g.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O

        eng = O.Engine(meta.as_dict(), {n: (t.shape, t.atom, t.data) for n, t in pk.tensors.items()}, REF_THREADS)
        sample = np.linspace(0, plen - 1, max(2, args.cpu_sample_steps // 2)).round().astype(np.int64)
        tok_s, dt = cpu_decode_rate(eng, sample, meta.vocab)
        line["cpu_baseline"] = {
            "value": tok_s, "unit": "tokens/s", "cores": REF_THREADS, "kind": "port",
            "sample": f"{sample.size} single-token steps at prompt positions {int(sample.min())}..{int(sample.max())} "
                      f"spread evenly ({dt:.1f} s; the reference prefills one token per step), oracle C++ "
                      f"restatement of the reference step, {REF_THREADS}-thread row split per matmul"}
    return line


def run_prefill(args, wl):
    world, rank, local, dev = dist_setup()
    line = measure_prefill(args, args.config, wl, world, rank, local, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch

        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------ tensor parallel
def tp_config(wl, world: int) -> dict:
    model, policy, batch, plen, dec, _s = wl
    return {"workload": "xl-int8-tp", "model": f"gpt2-{model}", "weights": policy, "global_batch": batch,
            "prompt": plen, "decode_positions": f"{plen}..{plen + dec - 1}",
            "parallelism": f"tp{world}" if world > 1 else "single GPU",
            "l2": "no flush: inputs larger than L2 (1.57 GB of int8 weights per step over the ranks)"}


def measure_tp(args, wl, world: int, rank: int, local: int, dev, parity: bool = False) -> dict:
    """GPT-2 XL int8, tensor parallel over the ranks; 16 sequences decoding positions 256..511.
    With `parity`, also compares a short greedy generation of the tensor-parallel handle with a
    1-GPU handle (rank 0) and with the oracle (rank 0)."""
    import torch

    from smelt_b200 import synth
    from smelt_b200.gpu import Gpu

    model, policy, batch, plen, dec, scaling = wl
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
    out = {}
    if parity:
        short = [ids[:TP_PARITY_PROMPT]]
        tp_tokens = g.generate_greedy(short, TP_PARITY_STEPS)[0]
        barrier(world)
        if rank == 0:
            with Gpu(pk, device=local, max_seqs=1) as g1:
                one_tokens = g1.generate_greedy(short, TP_PARITY_STEPS)[0]
            from oracle import oracle as O

            eng = O.Engine(meta.as_dict(), {n: (t.shape, t.atom, t.data) for n, t in pk.tensors.items()},
                           os.cpu_count() or 8)
            orc_tokens = eng.generate_greedy(short[0], TP_PARITY_STEPS)
            out["parity"] = {"prompt": TP_PARITY_PROMPT, "greedy_steps": TP_PARITY_STEPS,
                             "tp_tokens": tp_tokens.tolist(), "equal_to_1gpu": bool(np.array_equal(tp_tokens, one_tokens)),
                             "equal_to_oracle": bool(np.array_equal(tp_tokens, orc_tokens))}
            del eng
        barrier(world)
    g.prefill(prompts)
    done = 0
    for _ in range(max(args.warmup, 3)):
        g.decode_steps(1, batch, want_tokens=False)
        done += 1
    barrier(world)
    l0 = g.launches
    with ClockSampler(dev) as clk:
        timed_ms, k = 0.0, args.steps
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        while k > 0:
            if done >= dec:
                # prefills that rewind the positions are not decode steps: keep them out of the timing
                ev1.record(stream)
                torch.cuda.synchronize()
                timed_ms += ev0.elapsed_time(ev1)
                g.prefill(prompts)
                done = 0
                ev0.record(stream)
            n = min(k, dec - done)
            g.decode_steps(n, batch, want_tokens=False)
            done += n
            k -= n
        ev1.record(stream)
        torch.cuda.synchronize()
        timed_ms += ev0.elapsed_time(ev1)
    launches = g.launches - l0
    ms_max = max_over_ranks(timed_ms, world, dev)
    # each kernel's share of one decode step, from per-launch CUDA events in profiling mode (graphs
    # off); the tensor-parallel residual kernel's time includes its wait for the peers
    if done >= dec:
        g.prefill(prompts)
    g.profile(True)
    g.decode_steps(1, batch, want_tokens=False)
    prof = g.profile_read()
    g.profile(False)
    prof_total = sum(v["ms"] for v in prof.values()) or 1.0
    weights = sum(t.data.nbytes for t in pk.tensors.values() if len(t.shape) == 2)
    hbm, peak_kind = peaks()
    per_rank = weights / world / (ms_max / args.steps / 1e3) / 1e9
    out.update({
        "metric": METRICS["xl-int8-tp"], "value": batch * args.steps / (ms_max / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": "int8xfp32", "data": "synthetic", "config": tp_config(wl, world),
        "gpu_launches": int(launches), "clocks": clk.summary(),
        "kernels": {k: {"launches": v["launches"], "share_of_step": round(v["ms"] / prof_total, 4)}
                    for k, v in sorted(prof.items(), key=lambda kv: -kv[1]["ms"])[:8]},
        "tp_reduce_ln_share": round(prof.get("tp_reduce_ln", {"ms": 0.0})["ms"] / prof_total, 4),
        "roofline": {"bound": "hbm", "kernel": "whole decode step", "achieved": per_rank, "peak": hbm,
                     "unit": "GB/s", "frac": per_rank / hbm, "traffic": None, "peak_source": peak_kind,
                     "note": "weight bytes per rank only (KV excluded)"},
        "e2e": None,
    })
    g.close()
    return out


def run_tp(args, wl):
    world, rank, local, dev = dist_setup()
    line = measure_tp(args, wl, world, rank, local, dev, parity=world > 1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch

        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    wl = WORKLOADS[args.config]
    if args.batch > 0:
        wl = (wl[0], wl[1], args.batch) + tuple(wl[3:])
    if args.impl == "reference":
        run_reference(args, wl)
        return
    if args.config == "medium-int8-prefill":
        run_prefill(args, wl)
    elif args.config == "xl-int8-tp":
        run_tp(args, wl)
    elif args.config == "small-int8-trunk-bwd":
        run_trunk_bwd(args, wl)
    else:
        run_decode(args, wl)


if __name__ == "__main__":
    main()
