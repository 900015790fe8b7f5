"""SMT packer: HF GPT-2 weights (or seeded synthetic ones) -> SMT container.

The counterpart of the reference's converter binary (experiments/model-lab/src/bin/pack.rs):
it reads `config.json`, `tokenizer.json` and `model.safetensors` (F32) from a directory,
transposes the Conv1D weights to [out, in], applies the atom policy and writes the container
with the tokenizer embedded. `--synthetic small|medium|large|xl` packs the seeded N(0, 0.02)
weights used throughout this project instead.

    python -m smelt_b200.pack_smt assets --policy auto --out gpt2-q8.smt
    python -m smelt_b200.pack_smt --synthetic small --policy q4auto --out small-q4.smt
"""
from __future__ import annotations

import argparse
import json
import os
import struct
import sys

import numpy as np

from . import pack as P
from . import smt, synth


def read_safetensors(path: str) -> dict:
    """name -> float32 array of an F32 safetensors file (8-byte LE header length, JSON header,
    then the raw tensor bytes at the header's data_offsets)."""
    with open(path, "rb") as f:
        raw = f.read()
    (n,) = struct.unpack_from("<Q", raw, 0)
    header = json.loads(raw[8:8 + n])
    base = 8 + n
    out = {}
    for name, spec in header.items():
        if name == "__metadata__":
            continue
        if spec.get("dtype") != "F32":
            raise ValueError(f"{name}: dtype {spec.get('dtype')} (the packer reads F32 checkpoints)")
        o0, o1 = spec["data_offsets"]
        out[name] = np.frombuffer(raw, dtype="<f4", count=(o1 - o0) // 4, offset=base + o0).reshape(spec["shape"])
    return out


def meta_from_config(cfg: dict) -> P.Meta:
    return P.Meta(n_embd=int(cfg["n_embd"]), n_layer=int(cfg["n_layer"]), n_head=int(cfg["n_head"]),
                  n_ctx=int(cfg.get("n_ctx", cfg.get("n_positions", 1024))), vocab=int(cfg["vocab_size"]),
                  ln_eps=float(cfg.get("layer_norm_epsilon", 1e-5)))


def pack_dir(directory: str, policy: str):
    """(Pack, tokenizer bytes) from an HF GPT-2 directory."""
    with open(os.path.join(directory, "config.json")) as f:
        meta = meta_from_config(json.load(f))
    tok_path = os.path.join(directory, "tokenizer.json")
    tokenizer = open(tok_path, "rb").read() if os.path.exists(tok_path) else b"{}"
    tensors = read_safetensors(os.path.join(directory, "model.safetensors"))
    expected = P.hf_shapes(meta)
    hf = {}
    for name, shape in expected.items():
        key = name if name in tensors else "transformer." + name
        if key not in tensors:
            raise ValueError(f"missing tensor {name}")
        if tuple(tensors[key].shape) != tuple(shape):
            raise ValueError(f"{name}: shape {tuple(tensors[key].shape)}, expected {tuple(shape)}")
        hf[name] = tensors[key]
    return P.from_hf(meta, hf, policy), tokenizer


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("directory", nargs="?", help="HF GPT-2 directory (config.json, model.safetensors)")
    ap.add_argument("--synthetic", choices=sorted(P.CONFIGS), help="seeded synthetic weights instead")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--policy", default="auto", choices=P.POLICIES)
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    if bool(a.directory) == bool(a.synthetic):
        ap.error("give either a directory or --synthetic")
    if a.synthetic:
        pk = synth.synthetic_pack(P.CONFIGS[a.synthetic], a.policy, seed=a.seed)
        tokenizer = b"{}"
    else:
        pk, tokenizer = pack_dir(a.directory, a.policy)
    cid = smt.write_smt(a.out, pk, tokenizer)
    print(f"wrote {a.out}: {len(pk.tensors)} tensors, {os.path.getsize(a.out)} bytes, content_id {cid.hex()}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
