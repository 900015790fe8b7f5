"""Product-side atoms and converter against the oracle (bit-exact)."""
import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import atoms, pack as P, synth

from .helpers import TINY, hf, make_pack, oracle_engine


def edge_values(n_blocks=512, seed=3):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n_blocks * 32) * 0.02).astype(np.float32)
    x[:32] = 0.0                       # all-zero block
    x[32:64] *= 1e4                    # large values
    x[64:96] = 1e-30                   # subnormal scale territory
    x[96:128] = np.float32(127.5) * np.float32(0.001)  # round-half cases
    x[128:160] = -x[128:160]
    x[160:192] = np.linspace(-7, 7, 32)
    x[192:224] = 0.0
    x[200] = 1e-7                      # int4 scale rounds to f16 zero: 0/0 -> q = 0
    return x


@pytest.mark.parametrize("enc,oenc", [(atoms.q8_encode, O.q8_encode), (atoms.q4_encode, O.q4_encode),
                                      (atoms.q8_encode_fast, O.q8_encode), (atoms.q4_encode_fast, O.q4_encode)])
def test_encoders_bit_exact(enc, oenc):
    x = edge_values()
    assert np.array_equal(enc(x), oenc(x))


def test_f16_encode_bit_exact():
    x = edge_values()
    ours = atoms.f32_to_f16_bits(x)
    ref = np.array([O.f32_to_f16(float(v)) for v in x[:4096]], dtype=np.uint16)
    assert np.array_equal(ours[:4096], ref)


def test_rng_bit_exact():
    a = synth.Rng(0).normal_f32(300001, 0.02)
    b = O.Rng(0).normal_f32(300001, 0.02)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(synth.Rng(5).below(4096, 50257), O.Rng(5).below(4096, 50257))


@pytest.mark.parametrize("policy", ["auto", "q4auto", "core.f16", "f32", "core.i8.b32.f16scale"])
def test_converter_matches_oracle(policy):
    w = hf(TINY, 0, 0.02)
    pk = P.from_hf(TINY, w, policy)
    for name, t in pk.tensors.items():
        shp, atom, data = O.pack_tensor(name, w[name].shape, w[name], policy)
        assert shp == t.shape and atom == t.atom and np.array_equal(data, t.data), name


def test_atom_policy_and_transpose():
    pk = make_pack(TINY, "auto")
    d = TINY.n_embd
    assert pk.tensors["h.0.attn.c_attn.weight"].shape == (3 * d, d)
    assert pk.tensors["h.0.mlp.c_proj.weight"].shape == (d, 4 * d)
    assert pk.tensors["h.0.attn.c_attn.weight"].atom == atoms.ATOM_Q8
    assert pk.tensors["h.0.ln_1.weight"].atom == atoms.ATOM_F16
    assert pk.tensors["h.0.attn.c_attn.bias"].atom == atoms.ATOM_F16
    # transpose: packed row r of c_attn equals HF column r
    w = hf(TINY, 0, 0.0)["h.1.attn.c_attn.weight"]
    deq = pk.dequant("h.1.attn.c_attn.weight")
    q = atoms.dequant(atoms.ATOM_Q8, atoms.q8_encode(np.ascontiguousarray(w.T)), w.size).reshape(3 * d, d)
    assert np.array_equal(deq, q)


@pytest.mark.parametrize("policy", ["auto", "q4auto", "core.f16", "f32"])
def test_host_dequant_matches_oracle_vec_f32(policy):
    pk = make_pack(TINY, policy, 0, 0.02)
    eng = oracle_engine(pk)
    for name, t in pk.tensors.items():
        a = pk.dequant(name).reshape(-1)
        b = eng.vec_f32(name)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), name


def test_small_pack_sizes_match_reference_log():
    # model-lab.log:19 reports 126.0 MiB of active (2-D) Q8 bytes for GPT-2 small.
    shapes = P.hf_shapes(P.GPT2_SMALL)
    total = 0
    for name, s in shapes.items():
        if len(s) == 2:
            total += atoms.payload_bytes(P.choose_atom(s, "auto"), int(np.prod(s)))
    assert total == 132_088_368
    assert round(total / 2**20, 1) == 126.0
    assert len(shapes) == 148
