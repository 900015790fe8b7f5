"""SMT container (format.rs, gpt2.rs:43-110) and BLAKE3: the library's C++ reader and hash
against the committed BLAKE3 vectors and the oracle's Python restatement (oracle/smt_oracle.py),
round trips through write_smt, and refusal of any corrupted section or tensor. CPU only."""
import json
import os
import re
import struct

import numpy as np
import pytest

from oracle import smt_oracle
from smelt_b200 import _ffi, smt
from smelt_b200._ffi import Gpt2qError

from .golden.make_blake3 import data as golden_data
from .helpers import MINI, TINY, make_pack

HERE = os.path.dirname(__file__)
HEADER = os.path.join(HERE, "..", "include", "gpt2q.h")


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


def _vectors():
    with open(os.path.join(HERE, "golden", "blake3_vectors.json")) as f:
        return json.load(f)["vectors"]


def test_library_exports_every_declared_symbol():
    """Every function include/gpt2q.h declares is exported by libgpt2q.so and bound in _ffi."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    declared = set(re.findall(r"\b(gpt2q_\w+)\s*\(", text))
    assert declared == set(_ffi.EXPORTS)
    lib = _ffi.load()
    for name in sorted(declared):
        assert hasattr(lib, name), name


def test_blake3_native_matches_vectors():
    for v in _vectors():
        assert smt.blake3(golden_data(v["seed"], v["len"])).hex() == v["digest"], v["len"]


def test_blake3_restatement_matches_vectors():
    """The pure-Python restatement (small inputs only: it is slow)."""
    for v in _vectors():
        if v["len"] <= 70000:
            assert smt_oracle.blake3(golden_data(v["seed"], v["len"])).hex() == v["digest"], v["len"]


def test_blake3_matches_installed_binding_on_random_lengths():
    b3 = pytest.importorskip("blake3")
    rng = np.random.default_rng(11)
    for n in rng.integers(0, 40000, 40).tolist() + [int(x) for x in rng.integers(1 << 20, 5 << 20, 3)]:
        d = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert smt.blake3(d) == b3.blake3(d).digest(), n


def _sections(buf: bytes):
    off, out = 128, []
    while off < len(buf):
        ty, fl, ln = struct.unpack_from("<IIQ", buf, off)
        out.append((ty, fl, off + 16, ln))
        off += 16 + ln
    return out


def _remerkle(buf: bytearray) -> bytearray:
    """Recompute INDEX and the content_id after an edit, so only the tensor digests disagree."""
    secs = _sections(bytes(buf))
    digests = {}
    for ty, _, p, ln in secs:
        if ty != smt.SEC_INDEX:
            digests[ty] = smt.blake3(bytes(buf[p:p + ln]))
    for ty, _, p, ln in secs:
        if ty == smt.SEC_INDEX:
            index = b"".join(struct.pack("<I", t) + digests[t] for t, _, _, _ in secs if t != smt.SEC_INDEX)
            assert len(index) == ln
            buf[p:p + ln] = index
            digests[ty] = smt.blake3(index)
    buf[16:48] = smt.blake3(b"".join(sorted(digests.values())))
    return buf


@pytest.mark.parametrize("meta,policy", [(TINY, "auto"), (TINY, "q4auto"), (MINI, "core.f16"), (TINY, "f32")])
def test_write_then_inspect_and_read_round_trip(tmp_path, meta, policy):
    pk = make_pack(meta, policy)
    path = str(tmp_path / "m.smt")
    cid = smt.write_smt(path, pk)
    info = smt.inspect(path, verify=True)
    assert info["content_id"] == cid.hex() and info["verified"]
    a = info["arch"]
    assert (a["n_embd"], a["n_layer"], a["n_head"], a["n_ctx"], a["vocab_size"]) == (
        meta.n_embd, meta.n_layer, meta.n_head, meta.n_ctx, meta.vocab)
    assert [t["name"] for t in info["tensors"]] == list(pk.tensors)
    for t in info["tensors"]:
        ref = pk.tensors[t["name"]]
        assert t["atom"] == ref.atom and tuple(t["shape"]) == tuple(ref.shape) and t["len"] == ref.data.nbytes
    back = smt_oracle.read_smt(path)
    assert back.meta == pk.meta
    for name, t in pk.tensors.items():
        assert np.array_equal(back.tensors[name].data, np.ascontiguousarray(t.data).view(np.uint8).ravel())
    buf = open(path, "rb").read()
    assert struct.unpack_from("<H", buf, 4)[0] == smt.VERSION
    assert struct.unpack_from("<Q", buf, 48)[0] == len(buf)
    assert [s[0] for s in _sections(buf)] == [smt.SEC_META, smt.SEC_GRAPH, smt.SEC_TOKENIZER, smt.SEC_TENSORS,
                                              smt.SEC_INDEX]


def test_content_id_matches_installed_binding(tmp_path):
    """content_id = blake3 over the sorted section digests (format.rs:74-82), by the crate."""
    b3 = pytest.importorskip("blake3")
    path = str(tmp_path / "m.smt")
    cid = smt.write_smt(path, make_pack(TINY, "auto"))
    buf = open(path, "rb").read()
    digests = sorted(b3.blake3(buf[p:p + ln]).digest() for _, _, p, ln in _sections(buf))
    assert b3.blake3(b"".join(digests)).digest() == cid


def test_corruption_is_refused(tmp_path):
    pk = make_pack(TINY, "auto")
    path = str(tmp_path / "m.smt")
    smt.write_smt(path, pk)
    good = bytearray(open(path, "rb").read())
    secs = {ty: (p, ln) for ty, _, p, ln in _sections(bytes(good))}
    p_t, _ = secs[smt.SEC_TENSORS]
    json_len = struct.unpack_from("<I", good, p_t + 4)[0]
    recs = json.loads(good[p_t + 8:p_t + 8 + json_len])
    victim = recs[3]
    at = p_t + 8 + json_len + victim["offset"] + victim["len"] // 2

    def write(b, name):
        q = str(tmp_path / name)
        open(q, "wb").write(bytes(b))
        return q

    # a flipped payload byte breaks the merkle content_id
    bad = bytearray(good)
    bad[at] ^= 0x01
    q = write(bad, "flip.smt")
    with pytest.raises(Gpt2qError, match="merkle content_id mismatch"):
        smt.inspect(q, verify=True)
    smt.inspect(q, verify=False)  # without verification it parses
    with pytest.raises(ValueError, match="merkle"):
        smt_oracle.read_smt(q)
    # the same flip with INDEX and content_id recomputed: the tensor digest catches it
    q = write(_remerkle(bytearray(bad)), "flip_remerkle.smt")
    with pytest.raises(Gpt2qError, match="digest mismatch: " + re.escape(victim["name"])):
        smt.inspect(q, verify=True)
    with pytest.raises(ValueError, match="digest mismatch"):
        smt_oracle.read_smt(q)
    # a flipped META byte (inside the JSON) is a merkle mismatch too
    bad = bytearray(good)
    bad[secs[smt.SEC_META][0] + 3] ^= 0x20
    with pytest.raises(Gpt2qError, match="merkle"):
        smt.inspect(write(bad, "meta.smt"), verify=True)
    # bad magic, truncation, section length past the end
    bad = bytearray(good)
    bad[0:4] = b"SMT\x02"
    with pytest.raises(Gpt2qError, match="bad magic"):
        smt.inspect(write(bad, "magic.smt"), verify=False)
    with pytest.raises(Gpt2qError, match="past the end|truncated"):
        smt.inspect(write(good[:len(good) - 5], "trunc.smt"), verify=False)
    with pytest.raises(Gpt2qError, match="too short"):
        smt.inspect(write(good[:100], "short.smt"), verify=False)
    with pytest.raises(Gpt2qError, match="cannot open"):
        smt.inspect(str(tmp_path / "missing.smt"), verify=False)


def test_record_past_section_is_refused(tmp_path):
    """A tensor record whose offset+len leaves the TENSORS payload is refused even unverified."""
    pk = make_pack(TINY, "auto")
    path = str(tmp_path / "m.smt")
    smt.write_smt(path, pk)
    buf = bytearray(open(path, "rb").read())
    p_t, ln_t = {ty: (p, ln) for ty, _, p, ln in _sections(bytes(buf))}[smt.SEC_TENSORS]
    json_len = struct.unpack_from("<I", buf, p_t + 4)[0]
    text = buf[p_t + 8:p_t + 8 + json_len].decode()
    recs = json.loads(text)
    last = recs[-1]
    old = f'"offset": {last["offset"]}'
    new = f'"offset": {last["offset"] + 1}'.ljust(len(old))  # same JSON length: layout unchanged
    assert len(new) == len(old) and text.count(old) == 1
    buf[p_t + 8:p_t + 8 + json_len] = text.replace(old, new).encode()
    q = str(tmp_path / "past.smt")
    open(q, "wb").write(bytes(buf))
    with pytest.raises(Gpt2qError, match="runs past the section"):
        smt.inspect(q, verify=False)


def _write_safetensors(path, tensors: dict):
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        b = np.ascontiguousarray(arr, dtype="<f4").tobytes()
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
def test_packer_reads_hf_directory(tmp_path, policy):
    """pack_smt (the bin/pack.rs counterpart): config.json + model.safetensors + tokenizer.json
    -> SMT whose tensors equal the in-memory converter's and whose tokenizer is embedded."""
    from smelt_b200 import pack_smt

    from .helpers import hf
    meta = TINY
    d = tmp_path / "assets"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({"n_embd": meta.n_embd, "n_layer": meta.n_layer,
                                               "n_head": meta.n_head, "n_ctx": meta.n_ctx,
                                               "vocab_size": meta.vocab, "layer_norm_epsilon": 1e-5}))
    (d / "tokenizer.json").write_text('{"model": {"type": "BPE"}}')
    _write_safetensors(str(d / "model.safetensors"), hf(meta))
    out = str(tmp_path / "m.smt")
    assert pack_smt.main([str(d), "--policy", policy, "--out", out]) == 0
    info = smt.inspect(out, verify=True)
    assert info["verified"]
    back = smt_oracle.read_smt(out)
    ref = make_pack(meta, policy)
    assert back.meta == ref.meta
    for name, t in ref.tensors.items():
        assert back.tensors[name].atom == t.atom
        assert np.array_equal(back.tensors[name].data, np.ascontiguousarray(t.data).view(np.uint8).ravel()), name
    buf = open(out, "rb").read()
    tok = {ty: (p, ln) for ty, _, p, ln in _sections(buf)}[smt.SEC_TOKENIZER]
    assert buf[tok[0]:tok[0] + tok[1]] == b'{"model": {"type": "BPE"}}'
    with pytest.raises(SystemExit):
        pack_smt.main(["--out", out])  # neither a directory nor --synthetic


def test_unknown_sections_are_covered_by_the_merkle_but_ignored(tmp_path):
    """A section type the reader does not know (e.g. a future one) is hashed into the content_id
    like every other section (PackReader::verify walks all of them, format.rs:121-145) and
    otherwise ignored."""
    pk = make_pack(TINY, "auto")
    path = str(tmp_path / "m.smt")
    smt.write_smt(path, pk)
    buf = bytearray(open(path, "rb").read())
    extra = b"future section payload"
    buf += struct.pack("<IIQ", 99, 0, len(extra)) + extra
    # content_id over every section, the appended one included (INDEX itself is unchanged)
    digests = sorted(smt.blake3(bytes(buf[p:p + ln])) for _, _, p, ln in _sections(bytes(buf)))
    buf[16:48] = smt.blake3(b"".join(digests))
    buf[48:56] = struct.pack("<Q", len(buf))
    q = str(tmp_path / "extra.smt")
    open(q, "wb").write(bytes(buf))
    info = smt.inspect(q, verify=True)
    assert info["verified"] and len(info["tensors"]) == len(pk.tensors)
    # the same file without re-merkling fails verification
    bad = bytearray(open(path, "rb").read()) + struct.pack("<IIQ", 99, 0, len(extra)) + extra
    q2 = str(tmp_path / "extra_bad.smt")
    open(q2, "wb").write(bytes(bad))
    with pytest.raises(Gpt2qError, match="merkle"):
        smt.inspect(q2, verify=True)


def test_packer_synthetic_gpt2_small(tmp_path):
    """`python -m smelt_b200.pack_smt --synthetic small` writes a verifiable 148-tensor container."""
    from smelt_b200 import pack_smt

    out = str(tmp_path / "small.smt")
    assert pack_smt.main(["--synthetic", "small", "--policy", "auto", "--out", out]) == 0
    info = smt.inspect(out, verify=True)
    assert info["verified"] and len(info["tensors"]) == 148
    assert info["arch"] == {"n_embd": 768, "n_layer": 12, "n_head": 12, "n_ctx": 1024, "vocab_size": 50257}
    atoms = {t["name"]: t["atom"] for t in info["tensors"]}
    assert atoms["wte.weight"] == "core.i8.b32.f16scale" and atoms["ln_f.weight"] == "core.f16"


def test_missing_library_fails_loudly(tmp_path):
    """No fallback: without the built library every entry point refuses to load."""
    with pytest.raises(ImportError, match="not built"):
        _ffi.load(str(tmp_path / "libgpt2q.so"))
