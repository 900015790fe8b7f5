"""SMT container (v2-lite): writer, the library's reader/verifier, and BLAKE3.

Format (experiments/model-lab/src/format.rs:1-92, bin/pack.rs:119-150):

* 128-byte superheader: magic ``SMT\\x01``, version u16 = 2 at byte 4, the merkle content_id
  (32 bytes) at byte 16, the file length (u64) at byte 48.
* Sections from byte 128: ``type u32 | flags u32 | len u64 | payload``; META (2, JSON),
  GRAPH (3, JSON op list), TOKENIZER (4, bytes), TENSORS (5), then INDEX (1: ``type u32 ||
  blake3(payload)`` of every earlier section).
* TENSORS payload: ``[u32 count][u32 json_len][records JSON][tensor bytes]``; a record is
  ``{name, shape, atom, offset, len, digest}`` with offset relative to the tensor bytes and
  digest = the first 16 bytes of blake3(tensor bytes), lower-case hex.
* content_id = blake3 of the concatenated 32-byte section digests (every section, INDEX
  included) sorted bytewise.

Digests come from the library's BLAKE3 (``gpt2q_blake3``, smelt_b200/csrc/blake3.cpp); the
reader and verifier are the library's (``gpt2q_smt_inspect``, ``gpt2q_create_from_smt``).
"""
from __future__ import annotations

import ctypes as C
import json
import struct

import numpy as np

from . import _ffi
from .pack import Pack

MAGIC = b"SMT\x01"
VERSION = 2
SEC_INDEX, SEC_META, SEC_GRAPH, SEC_TOKENIZER, SEC_TENSORS = 1, 2, 3, 4, 5


def write_smt(path: str, pack: Pack, tokenizer: bytes = b"{}") -> bytes:
    """Write `pack` as an SMT container; returns its content_id."""
    meta = pack.meta
    recs, payload = [], bytearray()
    for name, t in pack.tensors.items():
        data = np.ascontiguousarray(t.data).view(np.uint8).tobytes()
        recs.append({"name": name, "shape": [int(x) for x in t.shape], "atom": t.atom,
                     "offset": len(payload), "len": len(data), "digest": blake3(data)[:16].hex()})
        payload += data
    meta_json = {"arch": {"name": "gpt2", "n_embd": meta.n_embd, "n_layer": meta.n_layer, "n_head": meta.n_head,
                          "n_ctx": meta.n_ctx, "vocab_size": meta.vocab, "ln_eps": meta.ln_eps},
                 "atom_manifest": {r["name"]: r["atom"] for r in recs}}
    graph = ["embed", "pos_add"]
    for l in range(meta.n_layer):
        graph += [f"h{l}.{op}" for op in ("ln_1", "attn.c_attn", "attn.mha_causal", "attn.c_proj", "resid",
                                          "ln_2", "mlp.c_fc", "gelu", "mlp.c_proj", "resid")]
    graph += ["ln_f", "tied_head"]
    recs_json = json.dumps(recs).encode()
    tensors = struct.pack("<II", len(recs), len(recs_json)) + recs_json + bytes(payload)
    sections = [(SEC_META, json.dumps(meta_json).encode()), (SEC_GRAPH, json.dumps(graph).encode()),
                (SEC_TOKENIZER, tokenizer), (SEC_TENSORS, tensors)]
    digests = [(ty, blake3(p)) for ty, p in sections]
    index = b"".join(struct.pack("<I", ty) + d for ty, d in digests)
    sections.append((SEC_INDEX, index))
    digests.append((SEC_INDEX, blake3(index)))
    content_id = blake3(b"".join(sorted(d for _, d in digests)))
    body = b"".join(struct.pack("<IIQ", ty, 0, len(p)) + p for ty, p in sections)
    header = bytearray(128)
    header[:4] = MAGIC
    header[4:6] = struct.pack("<H", VERSION)
    header[16:48] = content_id
    header[48:56] = struct.pack("<Q", 128 + len(body))
    with open(path, "wb") as f:
        f.write(bytes(header) + body)
    return content_id


def inspect(path: str, verify: bool = True) -> dict:
    """The library's parse (and verification) of an SMT file, as a dict; raises Gpt2qError."""
    lib = _ffi.load()
    buf = C.create_string_buffer(1 << 20)
    _ffi.check(lib, None, lib.gpt2q_smt_inspect(str(path).encode(), 1 if verify else 0, buf, len(buf)))
    return json.loads(buf.value.decode())


def blake3(data: bytes) -> bytes:
    """BLAKE3 computed by the library (gpt2q_blake3)."""
    lib = _ffi.load()
    out = (C.c_uint8 * 32)()
    src = bytes(data)
    _ffi.check(lib, None, lib.gpt2q_blake3(src, len(src), out))
    return bytes(out)
