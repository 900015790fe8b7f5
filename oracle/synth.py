"""Seeded synthetic GPT-2 models and token ids built by the oracle alone.

TEST INFRASTRUCTURE ONLY. The benchmark's reference arm and the tests use this to
obtain the workload's weights without loading the product library: every value
comes from the oracle's restatements,
  - Rng: xorshift64* of experiments/model-lab/src/gpu_backward.rs:835-856 with the
    Box-Muller normal of experiments/perf-lab/src/bin/atoms.rs:78-83 (orc_rng_*),
  - converter: Conv1D transpose and atom policy of
    experiments/model-lab/src/bin/pack.rs:47-84 (orc_pack_tensor).

Workload definition: every 2-D weight ~ N(0, 0.02); LayerNorm gain 1, bias 0;
linear biases 0, or N(0, bias_std) for the variant that exercises the bias adds.
Tensors are drawn from one Rng stream in sorted HF-name order, each filled in its
HF layout ([in, out] for Conv1D) before conversion, so the bytes equal the product
generator's (tests/test_oracle_synth.py checks that).
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

# HF GPT-2 configurations (experiments/model-lab/assets/config.json for small).
MODELS = {
    "small": dict(n_embd=768, n_layer=12, n_head=12, n_ctx=1024, vocab=50257, ln_eps=1e-5),
    "medium": dict(n_embd=1024, n_layer=24, n_head=16, n_ctx=1024, vocab=50257, ln_eps=1e-5),
    "xl": dict(n_embd=1600, n_layer=48, n_head=25, n_ctx=1024, vocab=50257, ln_eps=1e-5),
}


def hf_shapes(meta: dict) -> dict:
    """HF safetensors names and shapes of GPT-2, sorted by name (the converter's BTreeMap
    order, pack.rs:19,30)."""
    d, inter = meta["n_embd"], 4 * meta["n_embd"]
    s = {"wte.weight": (meta["vocab"], d), "wpe.weight": (meta["n_ctx"], d), "ln_f.weight": (d,),
         "ln_f.bias": (d,)}
    for layer in range(meta["n_layer"]):
        p = f"h.{layer}."
        s.update({p + "ln_1.weight": (d,), p + "ln_1.bias": (d,), p + "ln_2.weight": (d,), p + "ln_2.bias": (d,),
                  p + "attn.c_attn.weight": (d, 3 * d), p + "attn.c_attn.bias": (3 * d,),
                  p + "attn.c_proj.weight": (d, d), p + "attn.c_proj.bias": (d,),
                  p + "mlp.c_fc.weight": (d, inter), p + "mlp.c_fc.bias": (inter,),
                  p + "mlp.c_proj.weight": (inter, d), p + "mlp.c_proj.bias": (d,)})
    return dict(sorted(s.items()))


def _is_ln(name: str) -> bool:
    return ".ln_" in name or name.startswith("ln_")


def synthetic_tensors(meta: dict, policy: str = "auto", seed: int = 0, std: float = 0.02,
                      bias_std: float = 0.0) -> dict:
    """name -> (shape, atom, payload bytes) of the seeded model under `policy`
    ("auto", "q4auto", "core.f16", "core.i8.b32.f16scale" or "f32")."""
    rng = O.Rng(seed)
    out = {}
    for name, shape in hf_shapes(meta).items():
        n = int(np.prod(shape))
        if _is_ln(name):
            v = np.ones(n, np.float32) if name.endswith("weight") else np.zeros(n, np.float32)
        elif name.endswith("bias"):
            v = rng.normal_f32(n, bias_std) if bias_std > 0 else np.zeros(n, np.float32)
        else:
            v = rng.normal_f32(n, std)
        out[name] = O.pack_tensor(name, shape, v, policy)
    return out


def prompt_ids(n: int, vocab: int, seed: int = 1) -> np.ndarray:
    """Token ids uniform in [0, vocab) from Rng::below."""
    return O.Rng(seed).below(n, vocab)


def ragged_lengths(n_seq: int, lo: int, hi: int, seed: int = 2) -> np.ndarray:
    """Prompt lengths uniform in [lo, hi]."""
    return (O.Rng(seed).below(n_seq, hi - lo + 1) + lo).astype(np.int32)
