"""CUDA path vs the CPU oracle, through the C-ABI (libgpt2q.so via smelt_b200.gpu).

Acceptance (from the workload definition): dequantised weights bit-exact;
logits within 2e-2 max-abs with fp32 accumulation; identical greedy top-1
tokens (ties -> last index, gpt2.rs:390-396).
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import _ffi
from smelt_b200 import pack as P
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2  # max-abs logit tolerance for fp32 accumulation
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


@pytest.mark.parametrize("policy", ["auto", "q4auto", "core.f16", "f32"])
@pytest.mark.parametrize("meta", [TINY, MINI])
def test_dequant_bit_exact(meta, policy):
    pk = make_pack(meta, policy, 0, 0.02)
    eng = oracle_engine(pk)
    with Gpu(pk) as g:
        for name, t in pk.tensors.items():
            a = g.dequant(name, t.numel)
            b = eng.vec_f32(name)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), name


@pytest.mark.parametrize("policy", ["auto", "q4auto", "core.f16", "f32"])
def test_step_matches_golden(policy):
    gold = np.load(os.path.join(HERE, "golden", f"tiny_{policy.replace('.', '_')}.npz"))
    pk = make_pack(TINY, policy, 0, 0.02)
    with Gpu(pk) as g:
        got = np.stack([g.step(int(t), p) for p, t in enumerate(gold["ids"])])
        out = g.generate_greedy([gold["ids"][:8]], 16)[0]
    err = np.abs(got - gold["logits"]).max()
    assert err <= LOGIT_TOL, err
    assert np.array_equal(got.argmax(-1), gold["logits"].argmax(-1))
    assert np.array_equal(out, gold["greedy"])


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
@pytest.mark.parametrize("bias_std", [0.0, 0.02])
def test_step_matches_oracle_mini(policy, bias_std):
    pk = make_pack(MINI, policy, 0, bias_std)
    eng = oracle_engine(pk)
    ids = ((np.arange(40) * 101 + 7) % MINI.vocab).astype(np.uint32)
    ref = oracle_prefix_logits(eng, ids)
    with Gpu(pk) as g:
        got = np.stack([g.step(int(t), p) for p, t in enumerate(ids)])
        # clear_kv then replay: identical (Gpu::clear_kv, gpu.rs:203)
        g.clear_kv()
        again = np.stack([g.step(int(t), p) for p, t in enumerate(ids[:5])])
    err = np.abs(got - ref).max()
    assert err <= LOGIT_TOL, err
    assert err <= 1e-3, f"fp32 path drifted: {err}"
    assert np.array_equal(got[:5].view(np.uint32), again.view(np.uint32))
    assert all(O.argmax(got[i]) == O.argmax(ref[i]) for i in range(len(ids)))


@pytest.mark.parametrize("policy", ["auto", "q4auto", "f32"])
def test_prefill_and_decode_match_oracle(policy):
    pk = make_pack(MINI, policy, 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(11)
    lens = [1, 17, 64, 65, 100]
    prompts = [rng.integers(0, MINI.vocab, n).astype(np.uint32) for n in lens]
    with Gpu(pk, max_seqs=len(prompts), max_tokens=128) as g:
        nxt, lg = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(6, len(prompts))
    for i, p in enumerate(prompts):
        ref = oracle_prefix_logits(eng, p)[-1]
        assert np.abs(lg[i] - ref).max() <= LOGIT_TOL
        gen = eng.generate_greedy(p, 7)
        assert nxt[i] == gen[0]
        assert np.array_equal(toks[:, i], gen[1:7]), (i, toks[:, i], gen)


def test_batched_decode_is_batch_invariant():
    pk = make_pack(MINI, "auto", 0, 0.02)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, MINI.vocab, n).astype(np.uint32) for n in (9, 30, 2, 44)]
    with Gpu(pk, max_seqs=4) as g:
        g.prefill(prompts)
        batch = g.decode_steps(5, 4)
        singles = []
        for i, p in enumerate(prompts):
            g.prefill([p])
            singles.append(g.decode_steps(5, 1)[:, 0])
    for i in range(4):
        assert np.array_equal(batch[:, i], singles[i])


def test_decode_slots_and_positions():
    pk = make_pack(TINY, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    a = np.array([5, 6, 7, 8], np.uint32)
    b = np.array([50, 60], np.uint32)
    with Gpu(pk, max_seqs=3) as g:
        g.prefill([a[:3], b[:1]], slots=[2, 0])
        nxt, lg = g.decode([a[3], b[1]], [3, 1], slots=[2, 0], want_logits=True)
    ra = oracle_prefix_logits(eng, a)[-1]
    rb = oracle_prefix_logits(eng, b)[-1]
    assert np.abs(lg[0] - ra).max() <= LOGIT_TOL and np.abs(lg[1] - rb).max() <= LOGIT_TOL
    assert nxt[0] == O.argmax(ra) and nxt[1] == O.argmax(rb)


def test_errors_are_reported_and_handle_survives():
    pk = make_pack(TINY, "auto")
    with Gpu(pk, max_seqs=2) as g:
        with pytest.raises(_ffi.Gpt2qError) as e:
            g.step(TINY.vocab, 0)
        assert e.value.code == -1
        with pytest.raises(_ffi.Gpt2qError):
            g.step(1, TINY.n_ctx)
        with pytest.raises(_ffi.Gpt2qError):
            g.decode([1, 2], [0, 0], slots=[0, 0])
        with pytest.raises(_ffi.Gpt2qError):
            g.decode_steps(TINY.n_ctx + 1, 1)
        with pytest.raises(_ffi.Gpt2qError):
            g.dequant("no.such.tensor", 4)
        out = g.step(3, 0)
        assert np.isfinite(out).all()
    bad = P.Pack(TINY, dict(pk.tensors))
    del bad.tensors["h.1.mlp.c_fc.bias"]
    with pytest.raises(_ffi.Gpt2qError) as e:
        Gpu(bad)
    assert "h.1.mlp.c_fc.bias" in str(e.value)


def test_launch_counter_counts_graph_kernels():
    # fp32 weights take the per-kernel decode (the persistent decode needs int8)
    pk = make_pack(TINY, "f32")
    with Gpu(pk) as g:
        assert not g.info()["persistent_decode"]
        g.step(1, 0)
        n0 = g.launches
        g.step(2, 1)
        per_step = g.launches - n0
    # embed + 7 per layer + ln_f + head + argmax (partial + finalize)
    assert per_step == 1 + 7 * TINY.n_layer + 4


@pytest.mark.parametrize("policy", ["f32", "auto", "q4auto"])
def test_gpt2_small_greedy_64_matches_oracle(policy):
    """GPT-2 small, seed 0, prompt of 64 ids, 64 greedy steps: identical tokens."""
    from smelt_b200 import synth
    pk = make_pack(P.GPT2_SMALL, policy, 0, 0.0)
    prompt = synth.prompt_ids(64, P.GPT2_SMALL.vocab, seed=1)
    eng = oracle_engine(pk)
    ref = eng.generate_greedy(prompt, 64)
    with Gpu(pk) as g:
        got = g.generate_greedy([prompt], 64)[0]
        # per-token step path (Gpu::step usage in learn.rs) on the first 4 positions
        g.clear_kv()
        step_logits = np.stack([g.step(int(t), p) for p, t in enumerate(prompt[:4])])
    assert np.array_equal(got, ref), (got, ref)
    ref_logits = oracle_prefix_logits(eng, prompt[:4])
    assert np.abs(step_logits - ref_logits).max() <= LOGIT_TOL
