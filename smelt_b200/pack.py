"""GPT-2 weight pack: architecture metadata plus SMT tensor records.

Mirrors what LukasParke/smelt's converter writes into the TENSORS section
(experiments/model-lab/src/bin/pack.rs:28-95) and what Engine::load reads back
(experiments/model-lab/src/gpt2.rs:43-88): per tensor a name, an [out, in] shape
for 2-D weights (HF Conv1D weights are transposed at convert time, pack.rs:47-66),
an atom name and the payload bytes. The atom policy is pack.rs:68-84.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import atoms

CONV1D_SUFFIXES = ("attn.c_attn.weight", "attn.c_proj.weight", "mlp.c_fc.weight", "mlp.c_proj.weight")

# Policies: "auto" (reference default: Q8 for 2-D tensors with numel >= 4096, F16 otherwise),
# "core.f16" (everything F16), "core.i8.b32.f16scale" (every 2-D tensor Q8),
# "q4auto" (int4 where "auto" picks Q8), "f32" (fp32 weights throughout).
POLICIES = ("auto", atoms.ATOM_F16, atoms.ATOM_Q8, "q4auto", "f32")


@dataclass(frozen=True)
class Meta:
    """gpt2.rs:11-19."""
    n_embd: int
    n_layer: int
    n_head: int
    n_ctx: int
    vocab: int
    ln_eps: float = 1e-5

    def as_dict(self) -> dict:
        return dict(n_embd=self.n_embd, n_layer=self.n_layer, n_head=self.n_head, n_ctx=self.n_ctx,
                    vocab=self.vocab, ln_eps=self.ln_eps)


GPT2_SMALL = Meta(768, 12, 12, 1024, 50257)
GPT2_MEDIUM = Meta(1024, 24, 16, 1024, 50257)
GPT2_LARGE = Meta(1280, 36, 20, 1024, 50257)
GPT2_XL = Meta(1600, 48, 25, 1024, 50257)
CONFIGS = {"small": GPT2_SMALL, "medium": GPT2_MEDIUM, "large": GPT2_LARGE, "xl": GPT2_XL}


@dataclass
class Tensor:
    shape: tuple
    atom: str
    data: np.ndarray  # uint8 payload

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape))


@dataclass
class Pack:
    meta: Meta
    tensors: dict = field(default_factory=dict)  # name -> Tensor (insertion order = name order)

    def weight_bytes(self, two_d_only: bool = True) -> int:
        return sum(t.data.nbytes for t in self.tensors.values() if (len(t.shape) == 2 or not two_d_only))

    def dequant(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return atoms.dequant(t.atom, t.data, t.numel).reshape(t.shape)


def hf_shapes(meta: Meta, inter: int | None = None) -> dict:
    """HF safetensors names and shapes of GPT-2 (Conv1D weights are [in, out])."""
    d, inter = meta.n_embd, inter or 4 * meta.n_embd
    s = {"wte.weight": (meta.vocab, d), "wpe.weight": (meta.n_ctx, d),
         "ln_f.weight": (d,), "ln_f.bias": (d,)}
    for layer in range(meta.n_layer):
        p = f"h.{layer}."
        s.update({p + "ln_1.weight": (d,), p + "ln_1.bias": (d,), p + "ln_2.weight": (d,), p + "ln_2.bias": (d,),
                  p + "attn.c_attn.weight": (d, 3 * d), p + "attn.c_attn.bias": (3 * d,),
                  p + "attn.c_proj.weight": (d, d), p + "attn.c_proj.bias": (d,),
                  p + "mlp.c_fc.weight": (d, inter), p + "mlp.c_fc.bias": (inter,),
                  p + "mlp.c_proj.weight": (inter, d), p + "mlp.c_proj.bias": (d,)})
    return dict(sorted(s.items()))


def choose_atom(shape: tuple, policy: str) -> str:
    """pack.rs:68-84, plus the int4 and fp32 policies."""
    numel = int(np.prod(shape))
    two_d_big = numel >= 4096 and len(shape) == 2
    if policy == "f32":
        return atoms.ATOM_F32
    if policy == "auto" and two_d_big:
        return atoms.ATOM_Q8
    if policy == "q4auto" and two_d_big:
        return atoms.ATOM_Q4
    if policy in ("auto", "q4auto", atoms.ATOM_F16):
        return atoms.ATOM_F16
    if policy == atoms.ATOM_Q8 and len(shape) == 2:
        return atoms.ATOM_Q8
    return atoms.ATOM_F16


def convert_tensor(name: str, hf: np.ndarray, policy: str) -> Tensor:
    """One tensor through the converter: Conv1D transpose, then the atom policy."""
    f = np.ascontiguousarray(hf, dtype=np.float32)
    if f.ndim == 2 and name.endswith(CONV1D_SUFFIXES):
        f = np.ascontiguousarray(f.T)
    atom = choose_atom(f.shape, policy)
    if atom == atoms.ATOM_Q8:
        data = atoms.q8_encode_fast(f)
    elif atom == atoms.ATOM_Q4:
        data = atoms.q4_encode_fast(f)
    elif atom == atoms.ATOM_F32:
        data = f.reshape(-1).view(np.uint8).copy()
    else:
        data = atoms.f16_encode(f)
    return Tensor(tuple(int(s) for s in f.shape), atom, data)


def from_hf(meta: Meta, hf: dict, policy: str = "auto") -> Pack:
    """Convert HF-layout fp32 tensors (name -> array) into a Pack under `policy`."""
    if policy not in POLICIES:
        raise ValueError(f"unknown policy {policy}; one of {POLICIES}")
    pack = Pack(meta)
    for name in sorted(hf):
        pack.tensors[name] = convert_tensor(name, hf[name], policy)
    return pack
