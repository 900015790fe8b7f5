"""The tied lm head on the warp-level tensor cores (gemm_mma.cu k_head_mma) for 1..64 rows.

One CTA per SM stages the ln_f output's fp16 hi/lo pair once, and each warp runs whole 16-row
tiles of the int8 / int4 head weights over the full K: exact integer weights against x_hi and
x_lo, each group's fp32 sum scaled once, as in the layer linears. It serves decode batches and
the last rows of prefill where the tcgen05 head does not run (GPT2Q_HEAD_MMA=1, the default:
fewer than 16 rows), or for every 1..64 rows (GPT2Q_HEAD_MMA=2, forced here). Checked against the
heads it stands in for (GPT2Q_HEAD_MMA=0: the kind::i8 head below 16 rows, the tcgen05 f16 hi/lo
tile from 16) and the oracle's Engine::step
(experiments/model-lab/src/gpt2.rs:227-332, logits = wte . ln_f(x)), on vocabularies whose last
tile is ragged and CTAs of one or many tiles.
"""
import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import pack as P
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu
# 3001 rows: 188 tiles (two per CTA on some SMs), the last tile holding 9 rows
WIDE = P.Meta(n_embd=448, n_layer=2, n_head=7, n_ctx=96, vocab=3001)
# 20011 rows: 1251 tiles, about nine per CTA, every warp with one or two tiles; K = 6 groups
BIGV = P.Meta(n_embd=192, n_layer=1, n_head=3, n_ctx=64, vocab=20011)


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


def _run(pk, prompts, steps, monkeypatch, mode):
    monkeypatch.setenv("GPT2Q_HEAD_MMA", str(mode))
    monkeypatch.setenv("GPT2Q_NO_PERSISTENT", "1")  # one sequence decodes through the same head
    with Gpu(pk, max_seqs=len(prompts)) as g:
        nxt, lg0 = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(steps, len(prompts))
        nxt2, lg = g.decode(toks[-1], [p.size + steps for p in prompts], want_logits=True)
    return nxt, lg0, toks, nxt2, lg


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
@pytest.mark.parametrize("meta", [TINY, MINI, WIDE, BIGV], ids=["tiny", "mini", "wide", "bigv"])
@pytest.mark.parametrize("n_seq", [1, 5, 8, 17, 32, 64])
def test_warp_level_head_matches_other_heads_and_oracle(meta, policy, n_seq, monkeypatch):
    pk = make_pack(meta, policy, 0, 0.02)
    rng = np.random.default_rng(700 + n_seq)
    prompts = [rng.integers(0, meta.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, meta.n_ctx // 3, n_seq)]
    a = _run(pk, prompts, 3, monkeypatch, 2)
    b = _run(pk, prompts, 3, monkeypatch, 0)
    # both heads keep every product of the exact weights with the ~22-bit hi/lo activations
    assert np.abs(a[1] - b[1]).max() <= 1e-4 and np.abs(a[4] - b[4]).max() <= 1e-4
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])
    eng = oracle_engine(pk)
    for i in (0, n_seq - 1):
        ref = oracle_prefix_logits(eng, np.concatenate([prompts[i], [a[0][i]], a[2][:, i]]))
        p = prompts[i].size
        assert np.abs(a[1][i] - ref[p - 1]).max() <= 1e-3
        assert np.abs(a[4][i] - ref[-1]).max() <= 1e-3
        assert a[0][i] == O.argmax(ref[p - 1]) and a[3][i] == O.argmax(ref[-1])
        for s in range(3):
            assert a[2][s, i] == O.argmax(ref[p + s])


def test_warp_level_head_is_deterministic(monkeypatch):
    pk = make_pack(BIGV, "auto", 0, 0.02)
    rng = np.random.default_rng(17)
    prompts = [rng.integers(0, BIGV.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 20, 32)]
    x = _run(pk, prompts, 4, monkeypatch, 2)
    y = _run(pk, prompts, 4, monkeypatch, 2)
    for u, v in zip(x, y):
        assert np.array_equal(np.asarray(u).view(np.uint32), np.asarray(v).view(np.uint32))
