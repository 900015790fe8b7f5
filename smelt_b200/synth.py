"""Seeded synthetic GPT-2 weights and token ids (the benchmark workloads).

Weights follow the workload definition: every 2-D weight ~ N(0, 0.02), LayerNorm
gain 1 / bias 0, linear biases 0 (or N(0, bias_std) for the bias-exercising
variant). Values are drawn from one Rng stream in sorted tensor-name order, each
tensor filled in its HF layout ([in, out] for Conv1D) before conversion.

The Rng is model-lab's xorshift64* (experiments/model-lab/src/gpu_backward.rs:
835-856, Rng::new(seed) = seed ^ 0x9E3779B97F4A7C15) with the perf-lab Box-Muller
normal (experiments/perf-lab/src/bin/atoms.rs:78-83), implemented natively in
libgpt2q.so (gpt2q_rng_*).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _ffi
from .pack import POLICIES, Meta, Pack, convert_tensor, hf_shapes


class Rng:
    def __init__(self, seed: int):
        self._lib = _ffi.load()
        self.state = C.c_uint64(self._lib.gpt2q_rng_new(seed))

    def normal_f32(self, n: int, std: float) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self._lib.gpt2q_rng_normal_f32(C.byref(self.state), out.ctypes.data_as(_ffi._f32p), n, std)
        return out

    def below(self, n: int, bound: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint32)
        self._lib.gpt2q_rng_below(C.byref(self.state), out.ctypes.data_as(_ffi._u32p), n, bound)
        return out


def is_ln(name: str) -> bool:
    return ".ln_" in name or name.startswith("ln_")


def iter_hf_weights(meta: Meta, seed: int = 0, std: float = 0.02, bias_std: float = 0.0,
                    inter: int | None = None):
    """(name, HF-layout fp32 tensor) for `meta`, drawn in sorted-name order from Rng(seed)."""
    rng = Rng(seed)
    for name, shape in hf_shapes(meta, inter).items():
        n = int(np.prod(shape))
        if is_ln(name):
            v = np.ones(n, np.float32) if name.endswith("weight") else np.zeros(n, np.float32)
        elif name.endswith("bias"):
            v = rng.normal_f32(n, bias_std) if bias_std > 0 else np.zeros(n, np.float32)
        else:
            v = rng.normal_f32(n, std)
        yield name, v.reshape(shape)


def hf_weights(meta: Meta, seed: int = 0, std: float = 0.02, bias_std: float = 0.0,
               inter: int | None = None) -> dict:
    """HF-layout fp32 tensors for `meta`, drawn in sorted-name order from Rng(seed)."""
    return dict(iter_hf_weights(meta, seed, std, bias_std, inter))


def synthetic_pack(meta: Meta, policy: str = "auto", seed: int = 0, bias_std: float = 0.0) -> Pack:
    """The seeded model converted tensor by tensor (the fp32 copy of a large model is never
    held whole); equal to from_hf(meta, hf_weights(...), policy)."""
    if policy not in POLICIES:
        raise ValueError(f"unknown policy {policy}; one of {POLICIES}")
    pack = Pack(meta)
    for name, v in iter_hf_weights(meta, seed=seed, bias_std=bias_std):
        pack.tensors[name] = convert_tensor(name, v, policy)
    return pack


def prompt_ids(n: int, vocab: int, seed: int = 1) -> np.ndarray:
    """Token ids uniform in [0, vocab) from Rng::below."""
    return Rng(seed).below(n, vocab)


def ragged_lengths(n_seq: int, lo: int, hi: int, seed: int = 2) -> np.ndarray:
    """Prompt lengths uniform in [lo, hi]."""
    return (Rng(seed).below(n_seq, hi - lo + 1) + lo).astype(np.int32)
