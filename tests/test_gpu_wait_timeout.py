"""A bounded device-side wait that runs out is reported, and the handle stays usable.

The reference only panics when the GPU misbehaves (experiments/model-lab/src/gpu.rs:76,92).
Here every device-side wait is bounded. This test makes a real one run out, with no fault:
GPT2Q_TEST_SPLITK_STALL=1 at creation arms a one-shot switch in the tcgen05 linear. The
first split-K launch that reads it has the rank-1 CTA of a cluster withhold its partial sums,
so its peers' bounded mbarrier waits (2^26 polls, about a second) give up. The kernel still
completes every cluster-barrier phase and returns, and the host reports GPT2Q_ETIMEOUT. The next
prefill and decode on the same handle then give exactly what a fresh handle gives.
"""
import time

import numpy as np
import pytest

from smelt_b200 import _ffi
from smelt_b200 import pack as P
from smelt_b200 import synth
from smelt_b200.gpu import Gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


def test_split_k_wait_timeout_is_reported_and_the_handle_recovers(monkeypatch):
    pk = synth.synthetic_pack(P.GPT2_SMALL, "auto", seed=0)
    n, plen, steps = 32, 128, 4  # batched decode: d = 768 / 3072 linears run as split-K clusters
    ids = synth.prompt_ids(n * plen, pk.meta.vocab, seed=1)
    prompts = [ids[i * plen:(i + 1) * plen] for i in range(n)]
    # the decode linears of 32 tokens on the tcgen05 GEMM (whose split-K exchange has the wait)
    monkeypatch.setenv("GPT2Q_MMA_DISABLE", "1")
    with Gpu(pk, max_seqs=n) as clean:
        ref_next, ref_logits = clean.prefill(prompts, want_logits=True)
        ref_toks = clean.decode_steps(steps, n)
    monkeypatch.setenv("GPT2Q_TEST_SPLITK_STALL", "1")  # read when the handle is created
    g = Gpu(pk, max_seqs=n)
    monkeypatch.delenv("GPT2Q_TEST_SPLITK_STALL")
    try:
        assert g.info()["tensor_core"]
        t0 = time.perf_counter()
        with pytest.raises(_ffi.Gpt2qError) as e:
            g.prefill(prompts)
            g.decode_steps(steps, n)
        elapsed = time.perf_counter() - t0
        assert e.value.code == -5, e.value  # GPT2Q_ETIMEOUT
        assert "timed out" in str(e.value)
        assert elapsed < 120, elapsed  # the wait gave up instead of hanging
        # the same handle, after the error: identical to a handle that never saw it
        nxt, logits = g.prefill(prompts, want_logits=True)
        toks = g.decode_steps(steps, n)
        assert np.array_equal(nxt, ref_next)
        assert np.array_equal(logits.view(np.uint32), ref_logits.view(np.uint32))
        assert np.array_equal(toks, ref_toks)
    finally:
        g.close()
