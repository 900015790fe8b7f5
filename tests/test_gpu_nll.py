"""Teacher-forced NLL on the device (gpt2q_nll) vs the oracle's nll_per_token
(gpt2.rs:347-364): the head runs on every position and the log-sum-exp terms are formed
on the GPU; only the per-position f64 terms come back."""
import numpy as np
import pytest

from smelt_b200 import pack as P
from smelt_b200._ffi import Gpt2qError
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack, oracle_engine

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


@pytest.mark.parametrize("policy", ["auto", "q4auto", "f32"])
@pytest.mark.parametrize("meta", [TINY, MINI])
def test_nll_matches_oracle(meta, policy):
    pk = make_pack(meta, policy, 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(5)
    with Gpu(pk, max_seqs=2) as g:
        for n in (2, 17, meta.n_ctx):
            ids = rng.integers(0, meta.vocab, n).astype(np.uint32)
            got = g.nll(ids, slot=1)
            ref = eng.nll_per_token(ids)
            assert abs(got - ref) <= 2e-3 * max(1.0, abs(ref)), (n, got, ref)


LONG = P.Meta(n_embd=256, n_layer=2, n_head=4, n_ctx=512, vocab=1031)


def test_nll_long_sequence_chunks_and_errors():
    """300 positions: the head runs in two row chunks (256 + 43); bad arguments are refused."""
    pk = make_pack(LONG, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    ids = np.random.default_rng(9).integers(0, LONG.vocab, 300).astype(np.uint32)
    with Gpu(pk) as g:
        assert abs(g.nll(ids) - eng.nll_per_token(ids)) <= 2e-3
        with pytest.raises(Gpt2qError):
            g.nll(ids[:1])
        bad = ids.copy()
        bad[3] = MINI.vocab
        with pytest.raises(Gpt2qError):
            g.nll(bad)
