"""Post-ln_f plastic adapter h += B (A h) (Gpu::set_adapter gpu.rs:188-194,
k_adapter_apply cu/gpt2.cu:196-215) against the oracle's restatement, including an RCU-style
switch of generations between decode steps and clearing it."""
import numpy as np
import pytest

from smelt_b200.gpu import Gpu

from .helpers import MINI, make_pack, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


def _adapter(seed, r, d, scale=0.05):
    rng = np.random.default_rng(seed)
    return (rng.normal(0, scale, (r, d)).astype(np.float32), rng.normal(0, scale, (d, r)).astype(np.float32))


@pytest.mark.parametrize("policy", ["auto", "f32"])
def test_adapter_single_sequence_steps_match_oracle(policy):
    pk = make_pack(MINI, policy, 0, 0.02)
    eng = oracle_engine(pk)
    a, b = _adapter(1, 8, MINI.n_embd)
    eng.set_adapter(a, b)
    ids = ((np.arange(20) * 37 + 5) % MINI.vocab).astype(np.uint32)
    ref = oracle_prefix_logits(eng, ids)
    with Gpu(pk) as g:
        g.set_adapter(a, b)
        got = np.stack([g.step(int(t), p) for p, t in enumerate(ids)])
    assert np.abs(got - ref).max() <= TOL
    assert np.array_equal(got.argmax(-1), ref.argmax(-1))


def test_adapter_rcu_switch_and_clear_in_batched_decode():
    pk = make_pack(MINI, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, MINI.vocab, int(n)).astype(np.uint32) for n in (5, 17, 30)]
    gens = [_adapter(2, 16, MINI.n_embd), _adapter(3, 4, MINI.n_embd), None]
    with Gpu(pk, max_seqs=3) as g:
        nxt = g.prefill(prompts)
        fed = [list(p) + [int(t)] for p, t in zip(prompts, nxt)]
        got = []
        for gen in gens:  # two steps under each generation, then two without an adapter
            if gen is None:
                g.clear_adapter()
            else:
                g.set_adapter(*gen)
            for _ in range(2):
                nt, lg = g.decode([f[-1] for f in fed], [len(f) - 1 for f in fed], want_logits=True)
                got.append(lg)
                for f, t in zip(fed, nt):
                    f.append(int(t))
    # oracle: the same sequences, each step's logits under the adapter in force at that step
    for s in range(3):
        seq = np.array(fed[s], dtype=np.uint32)
        base = len(prompts[s]) + 1  # positions of the decode steps: base - 1 .. base + 4
        for k, gen in enumerate([gens[0], gens[0], gens[1], gens[1], None, None]):
            eng.set_adapter(*(gen if gen is not None else (None, None)))
            ref = oracle_prefix_logits(eng, seq[:base + k])[-1]
            assert np.abs(got[k][s] - ref).max() <= TOL, (s, k)


def test_adapter_on_the_persistent_single_sequence_path(monkeypatch):
    """With an adapter set, single-sequence decode stays on the persistent kernel (its head
    applies h += B(Ah) itself) and matches the per-kernel path and the oracle, step by step and
    across a multi-step launch; a generation switch between launches takes effect."""
    pk = make_pack(MINI, "auto", 0, 0.02)
    a, b = _adapter(3, 16, MINI.n_embd)
    a2, b2 = _adapter(4, 4, MINI.n_embd)
    ids = ((np.arange(12) * 29 + 3) % MINI.vocab).astype(np.uint32)
    eng = oracle_engine(pk)
    eng.set_adapter(a, b)
    ref = oracle_prefix_logits(eng, ids)
    with Gpu(pk) as g:
        if not g.info()["persistent_decode"]:
            pytest.skip("persistent decode not available: " + g.info()["persistent_why"])
        g.set_adapter(a, b)
        got = np.stack([g.step(int(t), p) for p, t in enumerate(ids)])
        assert np.abs(got - ref).max() <= TOL
        assert np.array_equal(got.argmax(-1), ref.argmax(-1))
        g.clear_kv()
        g.prefill([ids])
        multi = g.decode_steps(6, 1)[:, 0]
        g.set_adapter(a2, b2)
        after = g.decode_steps(3, 1)[:, 0]
    monkeypatch.setenv("GPT2Q_NO_PERSISTENT", "1")
    with Gpu(pk) as h:
        assert not h.info()["persistent_decode"]
        h.set_adapter(a, b)
        h.prefill([ids])
        ref_multi = h.decode_steps(6, 1)[:, 0]
        h.set_adapter(a2, b2)
        ref_after = h.decode_steps(3, 1)[:, 0]
    assert np.array_equal(multi, ref_multi)
    assert np.array_equal(after, ref_after)
