"""Persistent single-sequence decode (one launch for any number of steps) against the
per-kernel decode and the CPU oracle, through the C-ABI.

Acceptance as for every decode path: logits within 2e-2 max-abs of the oracle (observed
~1e-6), identical greedy tokens (ties -> last index, gpt2.rs:390-396).
"""
import os

import numpy as np
import pytest

from smelt_b200 import pack as P
from smelt_b200 import synth
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


def per_kernel_gpu(pk, **kw):
    """A handle created with the persistent decode switched off."""
    os.environ["GPT2Q_NO_PERSISTENT"] = "1"
    try:
        return Gpu(pk, **kw)
    finally:
        del os.environ["GPT2Q_NO_PERSISTENT"]


@pytest.mark.parametrize("meta", [TINY, MINI])
def test_eligibility_reported(meta):
    with Gpu(make_pack(meta, "auto")) as g:
        info = g.info()
        assert info["persistent_decode"], info
        assert info["persistent_ctas"] == 8 * meta.n_head
    for policy in ("f32", "q4auto"):
        with Gpu(make_pack(meta, policy)) as g:
            info = g.info()
            assert not info["persistent_decode"] and info["persistent_why"]
    with per_kernel_gpu(make_pack(meta, "auto")) as g:
        assert not g.info()["persistent_decode"]


@pytest.mark.parametrize("bias_std", [0.0, 0.02])
def test_step_logits_match_oracle_and_per_kernel(bias_std):
    pk = make_pack(MINI, "auto", 0, bias_std)
    eng = oracle_engine(pk)
    ids = ((np.arange(48) * 37 + 3) % MINI.vocab).astype(np.uint32)
    ref = oracle_prefix_logits(eng, ids)
    with Gpu(pk) as g:
        got = np.stack([g.step(int(t), p) for p, t in enumerate(ids)])
    with per_kernel_gpu(pk) as g:
        pk_got = np.stack([g.step(int(t), p) for p, t in enumerate(ids)])
    assert np.abs(got - ref).max() <= 1e-3
    assert np.abs(got - pk_got).max() <= 1e-3
    assert np.array_equal(got.argmax(-1), ref.argmax(-1))


def test_multi_step_launch_equals_single_steps():
    pk = make_pack(MINI, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    prompt = ((np.arange(30) * 11 + 1) % MINI.vocab).astype(np.uint32)
    with Gpu(pk) as g:
        g.prefill([prompt])
        n0 = g.launches
        many = g.decode_steps(40, 1)[:, 0]
        assert g.launches - n0 == 1  # 40 steps, one launch
        g.prefill([prompt])
        ones = np.array([g.decode_steps(1, 1)[0, 0] for _ in range(40)])
    ref = eng.generate_greedy(prompt, 41)[1:]
    assert np.array_equal(many, ones)
    assert np.array_equal(many, ref), (many, ref)


def test_context_edge_and_slots():
    """Positions up to n_ctx - 1, a non-zero slot, and the host-fed decode entry point."""
    pk = make_pack(TINY, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    prompt = ((np.arange(TINY.n_ctx - 10) * 7 + 2) % TINY.vocab).astype(np.uint32)
    with Gpu(pk, max_seqs=3) as g:
        g.prefill([prompt], slots=[2])
        toks = g.decode_steps(10, 1)[:, 0]  # last step runs at position n_ctx - 1
        nxt, lg = g.decode([toks[-2]], [TINY.n_ctx - 1], slots=[2], want_logits=True)
    ref = eng.generate_greedy(prompt, 11)
    assert np.array_equal(toks, ref[1:11])
    full = np.concatenate([prompt, ref[:10]])  # positions 0..n_ctx-1
    rl = oracle_prefix_logits(eng, full)[-1]
    assert np.abs(lg[0] - rl).max() <= LOGIT_TOL
    assert nxt[0] == ref[10]


def test_interleaves_with_batched_decode():
    """Single-sequence persistent steps and batched per-kernel steps share one KV arena."""
    pk = make_pack(MINI, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, MINI.vocab, n).astype(np.uint32) for n in (5, 19)]
    with Gpu(pk, max_seqs=2) as g:
        g.prefill(prompts)
        both = g.decode_steps(4, 2)
        g.prefill([prompts[1]], slots=[1])
        single = g.decode_steps(4, 1)[:, 0]
    for i, p in enumerate(prompts):
        assert np.array_equal(both[:, i], eng.generate_greedy(p, 5)[1:])
    assert np.array_equal(single, both[:, 1])


def test_gpt2_small_int8_greedy_64_persistent():
    """GPT-2 small int8, seed 0, 64-id prompt, 64 greedy steps in one persistent launch."""
    pk = make_pack(P.GPT2_SMALL, "auto", 0, 0.0)
    prompt = synth.prompt_ids(64, P.GPT2_SMALL.vocab, seed=1)
    eng = oracle_engine(pk)
    ref = eng.generate_greedy(prompt, 64)
    with Gpu(pk) as g:
        assert g.info()["persistent_decode"]
        g.prefill([prompt])
        n0 = g.launches
        got = g.decode_steps(63, 1)[:, 0]
        assert g.launches - n0 == 1
    assert np.array_equal(got, ref[1:]), (got, ref)
