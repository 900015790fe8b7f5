"""The tied lm head on kind::i8 (gemm.cu k_head_i8) for 1..64 rows with int8 head weights.

By default it runs below the tcgen05 head's 16 rows (instead of the CUDA-core GEMV);
GPT2Q_HEAD_I8=2 makes it run for every batch here, against GPT2Q_HEAD_I8=0 (never).

The ln_f output is split exactly into three int8 pieces per 32-group (k_head_pieces), the int8
weights enter unchanged, and the epilogue folds each group's exact integer products with the
weight and activation scales. Checked against the f16 hi/lo tensor-core head (GPT2Q_HEAD_I8=0) and
the oracle's Engine::step (experiments/model-lab/src/gpt2.rs:227-332), for decode batches that use
32 and 64 token slots, prompts whose last rows go through it at prefill, and an odd vocabulary.
"""
import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import pack as P
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu
WIDE = P.Meta(n_embd=448, n_layer=2, n_head=7, n_ctx=96, vocab=3001)  # 14 groups, 24 row tiles


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


def _run(pk, prompts, steps, monkeypatch, i8):
    monkeypatch.setenv("GPT2Q_HEAD_I8", "2" if i8 else "0")  # 2: every batch size, 0: never
    monkeypatch.setenv("GPT2Q_HEAD_MMA", "0")  # the comparison is with the f16 tensor-core head
    with Gpu(pk, max_seqs=len(prompts)) as g:
        nxt, lg0 = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(steps, len(prompts))
        nxt2, lg = g.decode(toks[-1], [p.size + steps for p in prompts], want_logits=True)
    return nxt, lg0, toks, nxt2, lg


@pytest.mark.parametrize("meta", [TINY, MINI, WIDE], ids=["tiny", "mini", "wide"])
@pytest.mark.parametrize("n_seq", [2, 17, 32, 40, 64])
def test_int8_head_matches_f16_head_and_oracle(meta, n_seq, monkeypatch):
    pk = make_pack(meta, "auto", 0, 0.02)
    rng = np.random.default_rng(500 + n_seq)
    prompts = [rng.integers(0, meta.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, meta.n_ctx // 3, n_seq)]
    a = _run(pk, prompts, 3, monkeypatch, True)
    b = _run(pk, prompts, 3, monkeypatch, False)
    # pieces keep ~20 bits of each group's largest value, the hi/lo split ~22: both far inside 1e-3
    assert np.abs(a[1] - b[1]).max() <= 1e-4 and np.abs(a[4] - b[4]).max() <= 1e-4
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])
    eng = oracle_engine(pk)
    for i in (0, n_seq - 1):
        ref = oracle_prefix_logits(eng, np.concatenate([prompts[i], [a[0][i]], a[2][:, i]]))
        p = prompts[i].size
        assert np.abs(a[1][i] - ref[p - 1]).max() <= 1e-3
        assert np.abs(a[4][i] - ref[-1]).max() <= 1e-3
        assert a[0][i] == O.argmax(ref[p - 1]) and a[3][i] == O.argmax(ref[-1])


def test_int8_head_is_deterministic_and_reports_its_launches(monkeypatch):
    pk = make_pack(MINI, "auto", 0, 0.02)
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, MINI.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 30, 24)]
    x = _run(pk, prompts, 4, monkeypatch, True)
    y = _run(pk, prompts, 4, monkeypatch, True)
    for u, v in zip(x, y):
        assert np.array_equal(np.asarray(u).view(np.uint32), np.asarray(v).view(np.uint32))
