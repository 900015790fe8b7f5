"""CUDA path vs the CPU oracle at the benchmark workloads' own shapes.

The kernels that produce the benchmarked numbers are checked here at the shapes they run,
against the oracle's restatement of Engine::step (experiments/model-lab/src/gpt2.rs:227-332):
  - GPT-2 small int8, 32 sequences x 128-token prompts, then decode through the batched
    tensor-core linears (d = 768 / 3072 split-K clusters) and the 393-tile lm head at M = 32;
  - GPT-2 small int4, 256 ragged prompts of 16..512 tokens (the shortest, the longest and
    two seeded others checked), then decode;
  - GPT-2 medium int8 (24 layers, d = 1024, 16 heads), 1024-token prompts: last-position
    logits and the greedy token;
  - GPT-2 XL int8 (48 layers, d = 1600, 25 heads) on one GPU, 16 sequences through the
    batched decode.
Inputs are the workloads' own seeded weights and token ids. The oracle side follows each
checked sequence greedily: its prompt through orc_engine_prefill (bit-identical to one
Engine::step per prompt token, tests/test_oracle_prefill.py), then one step per token.
Acceptance: logits within 2e-2 max-abs (and within what the handle's wide-tile products
achieve, tests/helpers.py TC_OBSERVED), identical greedy tokens (ties -> last index,
gpt2.rs:390-396).
"""
import functools

import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import pack as P
from smelt_b200 import synth
from smelt_b200.gpu import Gpu

from .helpers import observed

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2  # acceptance bound for fp32 accumulation


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


@functools.lru_cache(maxsize=2)
def pack(model: str, policy: str) -> P.Pack:
    return synth.synthetic_pack(P.CONFIGS[model], policy, seed=0)


def engine(pk: P.Pack) -> O.Engine:
    return O.Engine(pk.meta.as_dict(), {n: (t.shape, t.atom, t.data) for n, t in pk.tensors.items()}, 16)


def oracle_follow(eng: O.Engine, prompt, n_decode: int):
    """Greedy continuation: logits and argmax after the prompt and after each of n_decode steps."""
    kv = eng.empty_kv()
    lg = eng.prefill(prompt, kv)
    logits, toks = [lg], [O.argmax(lg)]
    for s in range(n_decode):
        lg = eng.step(toks[-1], len(prompt) + s, kv)
        logits.append(lg)
        toks.append(O.argmax(lg))
    return logits, toks


def gap(lg) -> float:
    top = np.sort(lg)[-2:]
    return float(top[1] - top[0])


def check_sequence(i, bound, ref_logits, ref_toks, got_first, got_first_tok, got_steps, got_last, got_last_tok):
    """got_steps[s] is the token the GPU predicted at decode step s (ref_toks[s + 1]); `bound` is
    the handle's observed accuracy (tests/helpers.py observed)."""
    for name, a, b in (("prompt", got_first, ref_logits[0]), ("last step", got_last, ref_logits[-1])):
        err = float(np.abs(a - b).max())
        assert err <= LOGIT_TOL, (i, name, err)
        assert err <= bound, (i, name, err)
    assert got_first_tok == ref_toks[0], (i, got_first_tok, ref_toks[0], gap(ref_logits[0]))
    for s, t in enumerate(got_steps):
        assert t == ref_toks[s + 1], (i, s, t, ref_toks[s + 1], gap(ref_logits[s + 1]))
    assert got_last_tok == ref_toks[-1], (i, got_last_tok, ref_toks[-1], gap(ref_logits[-1]))


def test_small_int8_batch32_decode():
    """The headline workload's shape: 32 x 128-token prompts, 8 decode steps, then logits."""
    pk = pack("small", "auto")
    V, n, plen, steps = pk.meta.vocab, 32, 128, 8
    ids = synth.prompt_ids(n * plen, V, seed=1)
    prompts = [ids[i * plen:(i + 1) * plen] for i in range(n)]
    with Gpu(pk, max_seqs=n) as g:
        assert g.info()["tensor_core"]
        bound = observed(g)
        nxt0, lg0 = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(steps, n)
        nxt, lg = g.decode(toks[-1], [plen + steps] * n, want_logits=True)
    eng = engine(pk)
    for i in (0, 7, 19, 31):
        ref_lg, ref_tok = oracle_follow(eng, prompts[i], steps + 1)
        check_sequence(i, bound, ref_lg, ref_tok, lg0[i], nxt0[i], toks[:, i], lg[i], nxt[i])


def test_small_int4_batch256_ragged_decode():
    """256 ragged prompts (16..512 tokens), 3 decode steps, then logits."""
    pk = pack("small", "q4auto")
    V, n, steps = pk.meta.vocab, 256, 3
    lens = synth.ragged_lengths(n, 16, 512, seed=2)
    ids = synth.prompt_ids(int(lens.sum()), V, seed=1)
    offs = np.concatenate([[0], np.cumsum(lens)])
    prompts = [ids[offs[i]:offs[i + 1]] for i in range(n)]
    with Gpu(pk, max_seqs=n, max_tokens=8192) as g:
        bound = observed(g)
        nxt0, lg0 = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(steps, n)
        nxt, lg = g.decode(toks[-1], (lens + steps).astype(np.int32), want_logits=True)
    eng = engine(pk)
    rng = np.random.default_rng(4)
    subset = sorted({int(np.argmin(lens)), int(np.argmax(lens)), *rng.choice(n, 2, replace=False).tolist()})
    for i in subset:
        ref_lg, ref_tok = oracle_follow(eng, prompts[i], steps + 1)
        check_sequence(i, bound, ref_lg, ref_tok, lg0[i], nxt0[i], toks[:, i], lg[i], nxt[i])


def test_medium_int8_prefill_1024():
    """Two of the prefill workload's 1024-token prompts: last-position logits and the next token."""
    pk = pack("medium", "auto")
    V, plen = pk.meta.vocab, 1024
    ids = synth.prompt_ids(64 * plen, V, seed=1)
    prompts = [ids[:plen], ids[plen:2 * plen]]
    with Gpu(pk, max_seqs=2, max_tokens=16384) as g:
        assert g.info()["tensor_core"]
        bound = observed(g)
        nxt, lg = g.prefill(prompts, want_logits=True)
    eng = engine(pk)
    for i, p in enumerate(prompts):
        ref = eng.prefill(p, eng.empty_kv())
        err = float(np.abs(lg[i] - ref).max())
        assert err <= LOGIT_TOL and err <= bound, (i, err)
        assert nxt[i] == O.argmax(ref), (i, nxt[i], O.argmax(ref), gap(ref))


def test_xl_int8_batch16_decode():
    """GPT-2 XL (25 heads, d = 1600) on one GPU: 16 sequences of 32 tokens, 4 decode steps."""
    pk = pack("xl", "auto")
    V, n, plen, steps = pk.meta.vocab, 16, 32, 4
    ids = synth.prompt_ids(n * 256, V, seed=1)
    prompts = [ids[i * 256:i * 256 + plen] for i in range(n)]
    with Gpu(pk, max_seqs=n) as g:
        bound = observed(g)
        nxt0, lg0 = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(steps, n)
        nxt, lg = g.decode(toks[-1], [plen + steps] * n, want_logits=True)
    eng = engine(pk)
    for i in (0, 15):
        ref_lg, ref_tok = oracle_follow(eng, prompts[i], steps + 1)
        check_sequence(i, bound, ref_lg, ref_tok, lg0[i], nxt0[i], toks[:, i], lg[i], nxt[i])
