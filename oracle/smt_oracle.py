"""Pure-Python restatement of the SMT container checks: BLAKE3 and the reader.

TEST INFRASTRUCTURE ONLY: the checker the library's C++ BLAKE3 and SMT reader
(smelt_b200/csrc/blake3.cpp, smt.cpp) are compared against. Only tests/ import it.

* ``blake3`` restates the published BLAKE3 specification (O'Connor, Aumasson, Neves,
  Wilcox-O'Hearn, 2020) in its recursive form; the reference calls the BLAKE3 team's Rust
  crate (model-lab Cargo.lock: blake3 1.8.7). Parity is pinned by digests of seeded inputs
  made with that crate's Python bindings (tests/golden/blake3_vectors.json).
* ``read_smt`` restates PackReader::open/verify/section (format.rs:94-175) and
  Engine::load + verify_tensor_digests (gpt2.rs:43-110).
"""
from __future__ import annotations

import json
import struct

import numpy as np

from smelt_b200.pack import Meta, Pack, Tensor

MAGIC = b"SMT\x01"
SEC_INDEX, SEC_META, SEC_GRAPH, SEC_TOKENIZER, SEC_TENSORS = 1, 2, 3, 4, 5

_IV = (0x6A09E667, 0xBB67AE85, 0x3C6EF372, 0xA54FF53A, 0x510E527F, 0x9B05688C, 0x1F83D9AB, 0x5BE0CD19)
_PERM = (2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8)
_CHUNK_START, _CHUNK_END, _PARENT, _ROOT = 1, 2, 4, 8
_M32 = 0xFFFFFFFF


def _rotr(x: int, n: int) -> int:
    return ((x >> n) | (x << (32 - n))) & _M32


def _g(s, a, b, c, d, mx, my):
    s[a] = (s[a] + s[b] + mx) & _M32
    s[d] = _rotr(s[d] ^ s[a], 16)
    s[c] = (s[c] + s[d]) & _M32
    s[b] = _rotr(s[b] ^ s[c], 12)
    s[a] = (s[a] + s[b] + my) & _M32
    s[d] = _rotr(s[d] ^ s[a], 8)
    s[c] = (s[c] + s[d]) & _M32
    s[b] = _rotr(s[b] ^ s[c], 7)


def _compress(cv, words, counter, block_len, flags):
    s = list(cv) + list(_IV[:4]) + [counter & _M32, (counter >> 32) & _M32, block_len, flags]
    m = list(words)
    for r in range(7):
        _g(s, 0, 4, 8, 12, m[0], m[1])
        _g(s, 1, 5, 9, 13, m[2], m[3])
        _g(s, 2, 6, 10, 14, m[4], m[5])
        _g(s, 3, 7, 11, 15, m[6], m[7])
        _g(s, 0, 5, 10, 15, m[8], m[9])
        _g(s, 1, 6, 11, 12, m[10], m[11])
        _g(s, 2, 7, 8, 13, m[12], m[13])
        _g(s, 3, 4, 9, 14, m[14], m[15])
        if r < 6:
            m = [m[i] for i in _PERM]
    return [s[i] ^ s[i + 8] for i in range(8)]


def _words(block: bytes):
    return list(struct.unpack("<16I", block.ljust(64, b"\0")))


def _chunk_node(chunk: bytes, counter: int):
    """(cv, last block words, block_len, flags) of a chunk before its final compression."""
    cv = list(_IV)
    blocks = [chunk[i:i + 64] for i in range(0, len(chunk), 64)] or [b""]
    for j, blk in enumerate(blocks[:-1]):
        cv = _compress(cv, _words(blk), counter, 64, _CHUNK_START if j == 0 else 0)
    last = blocks[-1]
    flags = _CHUNK_END | (_CHUNK_START if len(blocks) == 1 else 0)
    return cv, _words(last), counter, len(last), flags


def _subtree(data: bytes, first_chunk: int, root: bool):
    """Chaining value (or root bytes) of the left-complete subtree over `data`."""
    n_chunks = max(1, (len(data) + 1023) // 1024)
    if n_chunks == 1:
        cv, w, ctr, bl, fl = _chunk_node(data, first_chunk)
        return _compress(cv, w, ctr, bl, fl | (_ROOT if root else 0))
    left_chunks = 1 << ((n_chunks - 1).bit_length() - 1)  # largest power of two < n_chunks
    left = _subtree(data[:left_chunks * 1024], first_chunk, False)
    right = _subtree(data[left_chunks * 1024:], first_chunk + left_chunks, False)
    return _compress(list(_IV), left + right, 0, 64, _PARENT | (_ROOT if root else 0))


def blake3(data: bytes) -> bytes:
    """BLAKE3 hash, 32-byte output (recursive form of the specification's tree)."""
    return struct.pack("<8I", *_subtree(bytes(data), 0, True))


def read_smt(path: str, verify: bool = True) -> Pack:
    """Parse an SMT file into a Pack (PackReader + Engine::load, format.rs:94-175,
    gpt2.rs:43-110), checking the merkle content_id and every tensor digest with `blake3`
    above. Raises ValueError on a malformed file or a mismatch."""
    buf = open(path, "rb").read()
    if buf[:4] != MAGIC:
        raise ValueError("bad magic")
    sections, digests, off = {}, [], 128
    while off < len(buf):
        ty, _flags, ln = struct.unpack_from("<IIQ", buf, off)
        payload = buf[off + 16:off + 16 + ln]
        if len(payload) != ln:
            raise ValueError("section runs past the end of the file")
        sections.setdefault(ty, payload)
        if verify:
            digests.append(blake3(payload))
        off += 16 + ln
    if verify and blake3(b"".join(sorted(digests))) != buf[16:48]:
        raise ValueError("merkle content_id mismatch")
    arch = json.loads(sections[SEC_META])["arch"]
    meta = Meta(arch["n_embd"], arch["n_layer"], arch["n_head"], arch["n_ctx"], arch["vocab_size"],
                float(arch["ln_eps"]))
    sec = sections[SEC_TENSORS]
    count, json_len = struct.unpack_from("<II", sec, 0)
    recs = json.loads(sec[8:8 + json_len])
    if count != len(recs):
        raise ValueError("tensor count mismatch")
    base = 8 + json_len
    pack = Pack(meta)
    for r in recs:
        data = sec[base + r["offset"]:base + r["offset"] + r["len"]]
        if verify and blake3(data)[:16].hex() != r["digest"]:
            raise ValueError(f"digest mismatch: {r['name']}")
        pack.tensors[r["name"]] = Tensor(tuple(r["shape"]), r["atom"], np.frombuffer(data, dtype=np.uint8).copy())
    return pack
