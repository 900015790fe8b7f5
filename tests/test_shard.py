"""Host-side multi-GPU logic on CPU: sequence sharding with gloo ranks, and the
tensor-parallel split (heads / c_fc / c_proj) checked to reproduce the full forward."""
import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from smelt_b200 import shard
from smelt_b200 import pack as P

from .helpers import make_pack


def test_shard_sequences_partition_and_balance():
    rng = np.random.default_rng(0)
    lens = rng.integers(16, 513, 256)
    for world in (1, 2, 4, 8):
        parts = shard.shard_sequences(lens, world)
        assert parts[0][0] == 0 and parts[-1][1] == 256
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        loads = [lens[lo:hi].sum() for lo, hi in parts]
        assert max(loads) - min(loads) <= 2 * lens.max()


def _gloo_rank(rank, world, port, lens, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = shard.shard_sequences(lens, world)[rank]
    mine = list(range(lo, hi))
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    tokens = [int(sum(lens[i] for i in g)) for g in gathered]
    if rank == 0:
        out.put((gathered, tokens))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_cover_every_sequence_once():
    lens = list(np.random.default_rng(1).integers(16, 513, 37))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, lens, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, tokens = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    flat = sorted(i for g in gathered for i in g)
    assert flat == list(range(37))
    assert abs(tokens[0] - tokens[1]) <= 512


@pytest.mark.parametrize("tp", [2, 3, 4])
def test_tensor_parallel_split_reproduces_full_layer(tp):
    """Column split of c_attn by heads + row split of c_proj along K, summed over ranks
    (the all-reduce), equals the unsplit attention block output; same for the MLP."""
    meta = P.Meta(n_embd=320, n_layer=1, n_head=5, n_ctx=16, vocab=97)
    pk = make_pack(meta, "auto", 0, 0.02)
    d, hd = meta.n_embd, 64
    rng = np.random.default_rng(2)
    h = rng.standard_normal((3, d)).astype(np.float64)
    Wqkv = pk.dequant("h.0.attn.c_attn.weight").astype(np.float64)
    Wp = pk.dequant("h.0.attn.c_proj.weight").astype(np.float64)
    Wfc = pk.dequant("h.0.mlp.c_fc.weight").astype(np.float64)
    Wmp = pk.dequant("h.0.mlp.c_proj.weight").astype(np.float64)
    # attention-free check of the linear algebra: per-head values -> c_proj
    v_full = h @ Wqkv[2 * d:].T
    ref = v_full @ Wp.T
    acc = np.zeros_like(ref)
    covered = []
    for r in range(tp):
        h0, hn = shard.tp_heads(meta.n_head, tp, r)
        covered += list(range(h0, h0 + hn))
        rows = slice(2 * d + h0 * hd, 2 * d + (h0 + hn) * hd)
        acc += (h @ Wqkv[rows].T) @ Wp[:, h0 * hd:(h0 + hn) * hd].T
    assert covered == list(range(meta.n_head))
    np.testing.assert_allclose(acc, ref, rtol=1e-12, atol=1e-12)
    inter = Wfc.shape[0]
    if inter % (32 * tp) == 0:
        gelu = lambda v: 0.5 * v * (1 + np.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))
        ref2 = gelu(h @ Wfc.T) @ Wmp.T
        acc2 = np.zeros_like(ref2)
        for r in range(tp):
            f0, fn = shard.tp_fc_rows(inter, tp, r)
            acc2 += gelu(h @ Wfc[f0:f0 + fn].T) @ Wmp[:, f0:f0 + fn].T
        np.testing.assert_allclose(acc2, ref2, rtol=1e-12, atol=1e-12)
