"""Work partitioning across GPUs (one process per GPU).

Sequences are independent, so the batched configurations shard whole sequences
across ranks with no data-path collective; prompts are split into contiguous
ranges balanced by token count. The tensor-parallel split of GPT-2 XL mirrors
gpt2q_create_tp: whole heads per rank (the first n_head % tp ranks take one more),
c_fc rows and the c_proj K range in equal slices.
"""
from __future__ import annotations

import numpy as np


def shard_sequences(lengths, world: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) sequence ranges, one per rank, balancing total tokens."""
    lengths = np.asarray(lengths, dtype=np.int64)
    n = lengths.size
    if world <= 0:
        raise ValueError("world must be >= 1")
    csum = np.concatenate([[0], np.cumsum(lengths)])
    total = csum[-1]
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        i = int(np.searchsorted(csum, target))
        i = min(max(i, bounds[-1]), n)
        # keep at least one sequence for each remaining rank when possible
        i = min(i, n - (world - r)) if n >= world else i
        bounds.append(max(i, bounds[-1]))
    bounds.append(n)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def tp_heads(n_head: int, tp: int, rank: int) -> tuple[int, int]:
    """(first head, head count) of `rank` (gpt2q_create_tp)."""
    base, rem = divmod(n_head, tp)
    h0 = rank * base + min(rank, rem)
    return h0, base + (1 if rank < rem else 0)


def tp_fc_rows(inter: int, tp: int, rank: int) -> tuple[int, int]:
    """(first row, rows) of c_fc held by `rank` (and the matching mlp c_proj K range)."""
    if inter % (32 * tp):
        raise ValueError("c_fc rows must split into multiples of 32")
    per = inter // tp
    return rank * per, per
