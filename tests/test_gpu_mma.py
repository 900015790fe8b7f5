"""Warp-level tensor-core linear (mma.sync, gemm_mma.cu) for batched decode vs the oracle and vs
the two other linear paths.

Batched decode of 1..64 sequences runs the layer linears (q/k/v, attn c_proj, c_fc + GELU,
mlp c_proj) through this kernel by default (GPT2Q_MMA_MIN_M raises the lower bound; one
sequence alone takes the persistent kernel). GPT2Q_MMA_DISABLE=1 falls back to the tcgen05 GEMM
(16 tokens and up) and, with GPT2Q_TC_DISABLE=1 as well, to the CUDA-core kernel. All three must give the oracle's tokens
and logits within the split-precision bound; the mma path must be deterministic.
"""
import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import pack as P
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack, observed, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2
WIDE = P.Meta(n_embd=224 * 2, n_layer=2, n_head=7, n_ctx=96, vocab=3001)  # K = 448: 14 groups, 28 row tiles
# heads of 313 row tiles take the whole-tile layout; K = 6 and 10 groups are not multiples of the
# 8-group weight ring, so its refill runs on into the next tile mid-ring
HEAD6 = P.Meta(n_embd=192, n_layer=2, n_head=3, n_ctx=64, vocab=5003)
HEAD10 = P.Meta(n_embd=320, n_layer=1, n_head=5, n_ctx=64, vocab=5003)


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


MODES = {
    "mma": {"GPT2Q_MMA_DISABLE": "0", "GPT2Q_TC_DISABLE": "0"},
    "tc": {"GPT2Q_MMA_DISABLE": "1", "GPT2Q_TC_DISABLE": "0", "GPT2Q_TC_MIN_M": "16"},
    "simt": {"GPT2Q_MMA_DISABLE": "1", "GPT2Q_TC_DISABLE": "1"},
}


def _run(pk, prompts, steps, monkeypatch, mode, extra=None):
    for k, v in {**MODES[mode], **(extra or {})}.items():
        monkeypatch.setenv(k, v)
    with Gpu(pk, max_seqs=len(prompts)) as g:
        nxt, lg0 = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(steps, len(prompts))
        nxt2, lg = g.decode(toks[-1], [p.size + steps for p in prompts], want_logits=True)
        bounds[mode] = observed(g)  # prompts over 64 tokens in all go through the wide tiles
        tiles_per_cta[mode] = g.info()["mma_tiles_per_cta_max"]
    return nxt, lg0, toks, nxt2, lg


bounds = {}
tiles_per_cta = {}


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
@pytest.mark.parametrize("meta", [TINY, MINI, WIDE, HEAD6, HEAD10], ids=["tiny", "mini", "wide", "head6", "head10"])
@pytest.mark.parametrize("n_seq", [16, 17, 40, 64])
def test_mma_decode_matches_oracle_and_other_paths(meta, policy, n_seq, monkeypatch):
    pk = make_pack(meta, policy, 0, 0.02)
    rng = np.random.default_rng(n_seq)
    prompts = [rng.integers(0, meta.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, meta.n_ctx // 3, n_seq)]
    steps = 4
    res = {m: _run(pk, prompts, steps, monkeypatch, m) for m in MODES}
    a = res["mma"]
    bound = bounds["mma"]
    for other in ("tc", "simt"):
        b = res[other]
        assert np.abs(a[1] - b[1]).max() <= bound and np.abs(a[4] - b[4]).max() <= bound, other
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3]), other
    eng = oracle_engine(pk)
    for i in (0, n_seq - 1):
        ref = oracle_prefix_logits(eng, np.concatenate([prompts[i], [a[0][i]], a[2][:, i]]))
        p = prompts[i].size
        assert np.abs(a[1][i] - ref[p - 1]).max() <= bound
        assert np.abs(a[4][i] - ref[-1]).max() <= bound
        assert a[0][i] == O.argmax(ref[p - 1]) and a[3][i] == O.argmax(ref[-1])
        for s in range(steps):
            assert a[2][s, i] == O.argmax(ref[p + s])


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
@pytest.mark.parametrize("n_seq", [2, 5, 9])
def test_mma_for_few_tokens_matches_oracle(policy, n_seq, monkeypatch):
    """2..15-token decode steps through the warp-level kernel against the CUDA-core kernel."""
    pk = make_pack(MINI, policy, 0, 0.02)
    rng = np.random.default_rng(100 + n_seq)
    prompts = [rng.integers(0, MINI.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 40, n_seq)]
    a = _run(pk, prompts, 3, monkeypatch, "mma", {"GPT2Q_MMA_MIN_M": "1", "GPT2Q_NO_PERSISTENT": "1"})
    bound = bounds["mma"]
    b = _run(pk, prompts, 3, monkeypatch, "simt")
    assert np.abs(a[1] - b[1]).max() <= bound and np.abs(a[4] - b[4]).max() <= bound
    assert np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])


def test_mma_decode_is_deterministic_and_batch_invariant(monkeypatch):
    pk = make_pack(MINI, "auto", 0, 0.02)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, MINI.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 50, 32)]
    a = _run(pk, prompts, 5, monkeypatch, "mma")
    b = _run(pk, prompts, 5, monkeypatch, "mma")
    for x, y in zip(a, b):
        assert np.array_equal(np.asarray(x).view(np.uint32), np.asarray(y).view(np.uint32))


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
@pytest.mark.parametrize("meta", [MINI, WIDE], ids=["mini", "wide"])
def test_layernorm_applied_by_the_linear_matches_layernorm_launches(meta, policy, monkeypatch):
    """LN1 (from layer 1 on) and LN2 applied by the warp-level qkv / c_fc launches from the
    per-tile statistics that the residual linears write, against the same decode with the
    LayerNorm launches (GPT2Q_LN_FUSE=0): the same tokens, logits equal to rounding, and the
    oracle's logits within the bound."""
    pk = make_pack(meta, policy, 0, 0.02)
    rng = np.random.default_rng(77)
    prompts = [rng.integers(0, meta.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 12, 32)]
    fused = _run(pk, prompts, 6, monkeypatch, "mma")  # the decode steps of 32 tokens apply the LayerNorms
    plain = _run(pk, prompts, 6, monkeypatch, "mma", {"GPT2Q_LN_FUSE": "0"})
    assert np.abs(fused[1] - plain[1]).max() <= 1e-4 and np.abs(fused[4] - plain[4]).max() <= 1e-4
    assert np.array_equal(fused[0], plain[0]) and np.array_equal(fused[2], plain[2]) and np.array_equal(fused[3], plain[3])
    eng = oracle_engine(pk)
    for i in (0, 31):
        ref = oracle_prefix_logits(eng, np.concatenate([prompts[i], [fused[0][i]], fused[2][:, i]]))
        assert np.abs(fused[4][i] - ref[-1]).max() <= bounds["mma"]
        assert fused[3][i] == O.argmax(ref[-1])


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
@pytest.mark.parametrize("tiles,n_seq", [(2, 32), (3, 16), (5, 8), (8, 6)])
def test_multi_tile_layouts_match_one_tile(tiles, n_seq, policy, monkeypatch):
    """CTAs of 2, 3, 5 and 8 row tiles (GPT2Q_MMA_TILES), each tile a team of warps over one staged
    copy of the activations, against one tile per CTA (GPT2Q_MMA_MULTI=0). On WIDE, 3 and 5 tiles
    leave a ragged last CTA (112 c_fc tiles, 28 mlp c_proj tiles); the K-split clusters of the
    28-tile linears carry the tiles' partials too. The folded LayerNorms read and write their
    per-tile statistics through the same index arithmetic. Same tokens, logits within the bound,
    and the oracle's tokens and logits."""
    pk = make_pack(WIDE, policy, 0, 0.02)
    rng = np.random.default_rng(300 + tiles)
    prompts = [rng.integers(0, WIDE.vocab, int(n)).astype(np.uint32) for n in rng.integers(1, 30, n_seq)]
    few = {"GPT2Q_MMA_MIN_M": "1", "GPT2Q_NO_PERSISTENT": "1"}
    one = _run(pk, prompts, 4, monkeypatch, "mma", {**few, "GPT2Q_MMA_MULTI": "0"})
    assert tiles_per_cta["mma"] == 1
    monkeypatch.delenv("GPT2Q_MMA_MULTI")
    multi = _run(pk, prompts, 4, monkeypatch, "mma", {**few, "GPT2Q_MMA_TILES": str(tiles)})
    assert tiles_per_cta["mma"] == tiles
    bound = bounds["mma"]
    assert np.abs(one[1] - multi[1]).max() <= bound and np.abs(one[4] - multi[4]).max() <= bound
    assert np.array_equal(one[0], multi[0]) and np.array_equal(one[2], multi[2]) and np.array_equal(one[3], multi[3])
    eng = oracle_engine(pk)
    for i in (0, n_seq - 1):
        ref = oracle_prefix_logits(eng, np.concatenate([prompts[i], [multi[0][i]], multi[2][:, i]]))
        assert np.abs(multi[4][i] - ref[-1]).max() <= bound
        assert multi[3][i] == O.argmax(ref[-1])
