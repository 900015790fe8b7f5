"""Pins the oracle against the reference's own committed outputs and IEEE codecs.

tests/golden/atoms_log_ref.txt is docs/experiments/results/atoms.log:4-23 of
LukasParke/smelt: the perf-lab atom experiment's rms error and cosine for five
seeded distributions. Reproducing it digit for digit pins the f16 codec
(atoms.rs:10-61), the int4 atom math (perf-lab atoms.rs:89-99) and the perf-lab
RNG / Box-Muller the synthetic workloads use.
"""
import os

import numpy as np

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
DISTS = ["gauss01", "laplace_b1", "outlier_mix", "uniform_pm3", "tiny_gauss_1e-3"]
ATOMS = ["bf16_ref", "q4_sym_b32_f16scale", "mxfp4_e8m0_b32", "two_level_i4_sub16"]


def test_atoms_log_reproduced_exactly():
    ref = open(os.path.join(HERE, "golden", "atoms_log_ref.txt")).read().splitlines()
    r = O.perf_atoms(1 << 20)
    mine = [f"{d}, {a}, {r[i * 4 + j, 0]:.6f}, {r[i * 4 + j, 1]:.8f}"
            for i, d in enumerate(DISTS) for j, a in enumerate(ATOMS)]
    assert mine == ref


def test_f16_decode_exhaustive_matches_ieee():
    lib = O.lib()
    h = np.arange(65536, dtype=np.uint16)
    ours = np.array([lib.orc_f16_to_f32(int(v)) for v in h], dtype=np.float32)
    ieee = h.view(np.float16).astype(np.float32)
    fin = np.isfinite(ieee)
    assert np.array_equal(ours[fin].view(np.uint32), ieee[fin].view(np.uint32))
    assert np.all(np.isnan(ours[np.isnan(ieee)]))
    assert np.array_equal(np.isinf(ours), np.isinf(ieee))


def test_f16_encode_rne_matches_ieee():
    lib = O.lib()
    rng = np.random.default_rng(7)
    # random bit patterns spanning normals, subnormals, overflow and exact ties
    bits = rng.integers(0, 2**32, size=20000, dtype=np.uint64).astype(np.uint32)
    ties = (np.arange(1, 2000, dtype=np.uint32) << 13) | 0x1000 | (0x38000000)
    x = np.concatenate([bits.view(np.float32), ties.view(np.float32),
                        np.float32([0.0, -0.0, 65504, 65519.99, 65520, 1e-8, 6e-8, -3e-5])])
    x = x[np.isfinite(x)]
    ours = np.array([lib.orc_f32_to_f16(float(v)) for v in x], dtype=np.uint16)
    with np.errstate(over="ignore"):
        ieee = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ieee)


def test_q8_block_rules():
    x = np.zeros(96, np.float32)
    x[32:64] = np.linspace(-1, 1, 32)
    x[64:96] = 3.0
    b = O.q8_encode(x).reshape(3, 34)
    # zero block: scale 1.0 (f16 0x3c00), all q = 0
    assert b[0, 0] == 0x00 and b[0, 1] == 0x3C and not b[0, 2:].any()
    q = b[1, 2:].view(np.int8)
    assert q[0] == -127 and q[-1] == 127
    # q uses the unrounded fp32 scale: 3.0 / (3.0/127) rounds to 127 exactly
    assert np.all(b[2, 2:].view(np.int8) == 127)


def test_q4_block_rules():
    x = np.zeros(64, np.float32)
    x[32:64] = np.linspace(-0.7, 0.7, 32)
    b = O.q4_encode(x).reshape(2, 18)
    assert b[0, 0] == 0x00 and b[0, 1] == 0x3C and not b[0, 2:].any()
    lo = (b[1, 2:] & 0xF).astype(np.int8)
    hi = (b[1, 2:] >> 4).astype(np.int8)
    q = np.concatenate([lo, hi])
    q = np.where(q >= 8, q - 16, q)
    assert q[0] == -7 and q[31] == 7
    assert np.all(np.abs(q) <= 7)
