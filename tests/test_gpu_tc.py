"""Tensor-core (tcgen05) linear path vs the CPU oracle and vs the CUDA-core path.

GPT2Q_TC_MIN_M=1 forces every int8/int4 linear through the tcgen05 kernel (even
single-token decode); GPT2Q_TC_DISABLE=1 forces the CUDA-core kernel. Both are read
when a handle is created.
"""
import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import pack as P
from smelt_b200.gpu import Gpu

from .helpers import MINI, TC_OBSERVED, TINY, make_pack, observed, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
@pytest.mark.parametrize("meta", [TINY, MINI])
def test_tc_step_matches_oracle(meta, policy, monkeypatch):
    monkeypatch.setenv("GPT2Q_TC_MIN_M", "1")
    monkeypatch.setenv("GPT2Q_NO_PERSISTENT", "1")  # single-token steps through the tcgen05 linear
    pk = make_pack(meta, policy, 0, 0.02)
    eng = oracle_engine(pk)
    ids = ((np.arange(30) * 53 + 3) % meta.vocab).astype(np.uint32)
    ref = oracle_prefix_logits(eng, ids)
    with Gpu(pk) as g:
        got = np.stack([g.step(int(t), p) for p, t in enumerate(ids)])
    err = np.abs(got - ref).max()
    assert err <= LOGIT_TOL, err
    assert err <= 1e-3, f"tensor-core path less accurate than expected: {err}"
    assert np.array_equal(got.argmax(-1), ref.argmax(-1))


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
def test_tc_batched_decode_matches_cuda_core_path(policy, monkeypatch):
    pk = make_pack(MINI, policy, 0, 0.02)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, MINI.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 60, 40)]
    monkeypatch.setenv("GPT2Q_MMA_DISABLE", "1")  # 16..64 tokens would take the warp-level kernel
    res = {}
    for mode in ("simt", "tc"):
        monkeypatch.setenv("GPT2Q_TC_DISABLE", "1" if mode == "simt" else "0")
        monkeypatch.setenv("GPT2Q_TC_MIN_M", "16")
        with Gpu(pk, max_seqs=len(prompts)) as g:
            nxt, lg0 = g.prefill(prompts, want_logits=True)
            toks = g.decode_steps(8, len(prompts))
            nxt2, lg = g.decode(toks[-1], [p.size + 8 for p in prompts], want_logits=True)
            bound = observed(g)
        res[mode] = (nxt, lg0, toks, nxt2, lg)
    a, b = res["simt"], res["tc"]
    assert np.abs(a[1] - b[1]).max() <= bound
    assert np.abs(a[4] - b[4]).max() <= bound
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])


def test_tc_large_prefill_matches_oracle():
    pk = make_pack(MINI, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(9)
    lens = [128, 7, 100, 128, 33, 64, 128, 90, 1, 128, 128, 77, 55, 128, 128, 120]
    prompts = [rng.integers(0, MINI.vocab, n).astype(np.uint32) for n in lens]
    with Gpu(pk, max_seqs=len(prompts)) as g:
        nxt, lg = g.prefill(prompts, want_logits=True)
        bound = observed(g)
    for i in (0, 1, 8, 15):
        ref = oracle_prefix_logits(eng, prompts[i])[-1]
        assert np.abs(lg[i] - ref).max() <= bound
        assert nxt[i] == int(np.argmax(ref[::-1]) and (len(ref) - 1 - np.argmax(ref[::-1])))


LONG = P.Meta(n_embd=256, n_layer=2, n_head=4, n_ctx=512, vocab=1031)


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
def test_tc_prefill_attention_matches_cuda_cores_and_oracle(policy, monkeypatch):
    """Tensor-core prefill attention (128-query tiles, several 128-key blocks, ragged ends)
    against the CUDA-core attention kernel and the oracle."""
    pk = make_pack(LONG, policy, 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(7)
    lens = [1, 127, 128, 129, 300, 450]
    prompts = [rng.integers(0, LONG.vocab, n).astype(np.uint32) for n in lens]
    with Gpu(pk, max_seqs=len(prompts), max_tokens=2048) as g:
        nxt_tc, lg_tc = g.prefill(prompts, want_logits=True)
        bound = observed(g)
    monkeypatch.setenv("GPT2Q_ATTN_CORES", "1")
    with Gpu(pk, max_seqs=len(prompts), max_tokens=2048) as g:
        nxt_cc, lg_cc = g.prefill(prompts, want_logits=True)
    assert np.abs(lg_tc - lg_cc).max() <= 1e-3  # same linears: only the attention kernels differ
    assert np.array_equal(nxt_tc, nxt_cc)
    for i, p in enumerate(prompts):
        ref = oracle_prefix_logits(eng, p)[-1]
        assert np.abs(lg_tc[i] - ref).max() <= bound
        assert nxt_tc[i] == O.argmax(ref)


MID = P.Meta(n_embd=384, n_layer=2, n_head=6, n_ctx=128, vocab=1031)


@pytest.mark.parametrize("batch", [17, 40, 64, 100, 200])
def test_tc_split_k_exchange_shapes_match_cuda_core_path(batch, monkeypatch):
    """d = 384 decode batches split K 3 to 16 ways; at 33-64 sequences some reducing CTAs own
    a narrower last block of token columns than the others (e.g. 12, 12, 12, 12, 12, 4); at 100
    and 200 sequences the 128- and 256-token tiles exchange their partials the same way."""
    pk = make_pack(MID, "auto", 1, 0.02)
    rng = np.random.default_rng(batch)
    prompts = [rng.integers(0, MID.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 50, batch)]
    monkeypatch.setenv("GPT2Q_MMA_DISABLE", "1")  # keep the tcgen05 split-K tiles on the decode path
    res = {}
    for mode in ("simt", "tc"):
        monkeypatch.setenv("GPT2Q_TC_DISABLE", "1" if mode == "simt" else "0")
        with Gpu(pk, max_seqs=batch) as g:
            g.prefill(prompts)
            toks = g.decode_steps(4, batch)
            nxt, lg = g.decode(toks[-1], [p.size + 4 for p in prompts], want_logits=True)
            bound = observed(g)
        res[mode] = (toks, nxt, lg)
    a, b = res["simt"], res["tc"]
    assert np.abs(a[2] - b[2]).max() <= bound
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_persistent_prefill_gemm_matches_per_tile_launch(monkeypatch):
    """4096 prompt tokens: the 1024-row c_fc (8 x 16 = 128 tiles) runs in the persistent form
    (one CTA per SM walking tiles, double-buffered TMEM accumulator). Same MMAs in the same
    order as the one-tile-per-CTA launch, so the logits must be identical; and the oracle agrees."""
    pk = make_pack(MINI, "auto", 0, 0.02)
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, MINI.vocab, 128).astype(np.uint32) for _ in range(32)]
    res = {}
    for mode in ("persistent", "per_tile"):
        monkeypatch.setenv("GPT2Q_TC_NO_PERSISTENT", "1" if mode == "per_tile" else "")
        if mode == "persistent":
            monkeypatch.delenv("GPT2Q_TC_NO_PERSISTENT")
        with Gpu(pk, max_seqs=len(prompts), max_tokens=4096) as g:
            res[mode] = g.prefill(prompts, want_logits=True)
            bound = observed(g)
    assert np.array_equal(res["persistent"][0], res["per_tile"][0])
    assert np.array_equal(res["persistent"][1], res["per_tile"][1])
    eng = oracle_engine(pk)
    for i in (0, 31):
        ref = oracle_prefix_logits(eng, prompts[i])[-1]
        assert np.abs(res["persistent"][1][i] - ref).max() <= bound


@pytest.mark.parametrize("products", [1, 2, 3])
@pytest.mark.parametrize("policy", ["auto", "q4auto"])
def test_wide_tile_products_against_oracle(products, policy, monkeypatch):
    """GPT2Q_TC_PRODUCTS selects the MMAs of the wide tiles (prefill, and decode batches over 64
    tokens): 1 = W_hi X_hi, 2 = + W_lo X_hi (the exact weights), 3 = + W_hi X_lo (the default).
    Each holds the 2e-2 bound and its own observed bound through a 4096-token prefill
    (persistent form) and decode steps of 100 sequences (split-K wide tiles). Every greedy token
    equals the oracle's, evaluated on the GPU's own history, where the oracle's top-2 gap is
    wider than twice the variant's bound (inside it a reduced-precision variant may flip)."""
    monkeypatch.setenv("GPT2Q_TC_PRODUCTS", str(products))
    pk = make_pack(MINI, policy, 0, 0.02)
    eng = oracle_engine(pk)
    rng = np.random.default_rng(31)
    prompts = [rng.integers(0, MINI.vocab, int(n)).astype(np.uint32) for n in rng.integers(20, 80, 100)]
    with Gpu(pk, max_seqs=len(prompts), max_tokens=8192) as g:
        assert g.info()["tc_products"] == products
        nxt, lg0 = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(4, len(prompts))
        nxt2, lg = g.decode(toks[-1], [p.size + 4 for p in prompts], want_logits=True)
    for i in (0, 57, 99):
        p = prompts[i]
        ref = oracle_prefix_logits(eng, np.concatenate([p, [nxt[i]], toks[:, i]]))
        for got, r in ((lg0[i], ref[p.size - 1]), (lg[i], ref[-1])):
            err = float(np.abs(got - r).max())
            assert err <= LOGIT_TOL and err <= TC_OBSERVED[products], (i, err)
        picks = [(nxt[i], ref[p.size - 1]), (nxt2[i], ref[-1])] + [(toks[s, i], ref[p.size + s]) for s in range(4)]
        for t, r in picks:
            top2 = np.sort(r)[-2:]
            if products == 3 or top2[1] - top2[0] > 2 * TC_OBSERVED[products]:
                assert t == O.argmax(r), (i, t, O.argmax(r), top2)
