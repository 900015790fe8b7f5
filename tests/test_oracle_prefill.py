"""The oracle's batched prefill (orc_engine_prefill) is bit-identical to one Engine::step per
prompt token (gpt2.rs:227-332 driven by gpt2.rs:373-381): logits of the last position and every
K/V row, on every atom, with and without biases and an adapter, continuing from a partly filled
cache, and on widths that exercise the GEMV tails (columns not a multiple of 128)."""
import numpy as np
import pytest

from smelt_b200 import pack as P

from .helpers import MINI, TINY, make_pack, oracle_engine

WIDE_TAIL = P.Meta(n_embd=224, n_layer=2, n_head=2, n_ctx=40, vocab=101)  # 7 groups: 4 + a 3-group tail
NARROW = P.Meta(n_embd=96, n_layer=2, n_head=3, n_ctx=24, vocab=67)       # 3 groups: tail only


def _same(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


@pytest.mark.parametrize("policy", ["auto", "q4auto", "core.f16", "f32"])
@pytest.mark.parametrize("meta", [TINY, MINI, WIDE_TAIL, NARROW], ids=["tiny", "mini", "wide_tail", "narrow"])
def test_prefill_equals_per_token_steps(meta, policy):
    pk = make_pack(meta, policy, 0, 0.02)
    eng = oracle_engine(pk)
    ids = ((np.arange(meta.n_ctx - 2) * 37 + 5) % meta.vocab).astype(np.uint32)
    kv1 = eng.empty_kv()
    for p, t in enumerate(ids):
        ref = eng.step(int(t), p, kv1)
    kv2 = eng.empty_kv()
    split = len(ids) // 3
    eng.prefill(ids[:split], kv2)
    got = eng.prefill(ids[split:], kv2, pos0=split)
    assert _same(got, ref)
    assert _same(kv1, kv2)


def test_prefill_applies_the_adapter_like_step():
    pk = make_pack(MINI, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(3)
    eng.set_adapter(rng.normal(0, 0.05, (4, MINI.n_embd)).astype(np.float32),
                    rng.normal(0, 0.05, (MINI.n_embd, 4)).astype(np.float32))
    ids = ((np.arange(20) * 11 + 2) % MINI.vocab).astype(np.uint32)
    kv1 = eng.empty_kv()
    for p, t in enumerate(ids):
        ref = eng.step(int(t), p, kv1)
    assert _same(eng.prefill(ids, eng.empty_kv()), ref)


def test_prefill_rejects_bad_arguments():
    pk = make_pack(TINY, "auto")
    eng = oracle_engine(pk)
    with pytest.raises(ValueError):
        eng.prefill(np.array([TINY.vocab], np.uint32), eng.empty_kv())
    with pytest.raises(ValueError):
        eng.prefill(np.zeros(4, np.uint32), eng.empty_kv(), pos0=TINY.n_ctx - 3)
