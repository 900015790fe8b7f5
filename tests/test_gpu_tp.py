"""Tensor-parallel handles (gpt2q_create_tp, partial sums read from peer memory) on 2 GPUs vs one GPU.

A 5-head model splits unevenly (3 + 2 heads), like GPT-2 XL's 25 heads over 2/4/8
ranks. Ranks run as spawned processes, one per GPU; NVLS is off for the test.
"""
import os

import numpy as np
import pytest

from smelt_b200 import pack as P

from .helpers import make_pack

pytestmark = pytest.mark.gpu
META5 = P.Meta(n_embd=320, n_layer=2, n_head=5, n_ctx=128, vocab=1031)


def _prompts():
    rng = np.random.default_rng(7)
    return [rng.integers(0, META5.vocab, n).astype(np.uint32) for n in (9, 40)]


def _rank(rank, world, uid, policy, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    torch.cuda.set_device(rank)
    from smelt_b200.gpu import Gpu

    pk = make_pack(META5, policy, 0, 0.02)
    try:
        with Gpu(pk, device=rank, max_seqs=2, tp_size=world, tp_rank=rank, nccl_id=uid) as g:
            nxt, lg = g.prefill(_prompts(), want_logits=True)
            toks = g.decode_steps(5, 2)
            nxt2, lg2 = g.decode(toks[-1], [p.size + 5 for p in _prompts()], want_logits=True)
            peer = g.info()["tp_peer_mapped"]
        q.put((rank, None, nxt, lg, toks, nxt2, lg2, peer))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None, None, None, None, None, None))


@pytest.mark.parametrize("policy", ["auto", "q4auto"])
def test_tp2_matches_single_gpu(policy):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from smelt_b200 import build

    build.build()
    from smelt_b200.gpu import Gpu

    pk = make_pack(META5, policy, 0, 0.02)
    with Gpu(pk, device=0, max_seqs=2) as g:
        nxt, lg = g.prefill(_prompts(), want_logits=True)
        toks = g.decode_steps(5, 2)
        nxt2, lg2 = g.decode(toks[-1], [p.size + 5 for p in _prompts()], want_logits=True)
    uid = torch.cuda.nccl.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, policy, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=300)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=120)
    for r in (0, 1):
        assert res[r][1] is None, res[r][1]
        _, _, n_r, lg_r, t_r, n2_r, lg2_r, peer = res[r]
        assert peer, "NVLink-connected GPUs: the partials are summed from peer memory"
        assert np.abs(lg_r - lg).max() <= 1e-3
        assert np.abs(lg2_r - lg2).max() <= 1e-3
        assert np.array_equal(n_r, nxt) and np.array_equal(t_r, toks) and np.array_equal(n2_r, nxt2)
    # and the oracle's own greedy continuation (Engine::step, gpt2.rs:227-332)
    from oracle import oracle as O

    from .helpers import oracle_engine, oracle_prefix_logits

    eng = oracle_engine(pk)
    _, _, n_r, lg_r, t_r, n2_r, lg2_r, _ = res[0]
    for i, p in enumerate(_prompts()):
        seq = np.concatenate([p, [n_r[i]], t_r[:, i]])
        ref = oracle_prefix_logits(eng, seq)
        assert np.abs(lg_r[i] - ref[p.size - 1]).max() <= 1e-3
        assert np.abs(lg2_r[i] - ref[-1]).max() <= 1e-3
        assert n_r[i] == O.argmax(ref[p.size - 1]) and n2_r[i] == O.argmax(ref[-1])
        for s in range(t_r.shape[0]):
            assert t_r[s, i] == O.argmax(ref[p.size + s])
