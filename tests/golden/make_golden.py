"""Generate the committed golden fixtures from the CPU oracle.

    python tests/golden/make_golden.py

Writes tests/golden/tiny_<policy>.npz: for the seeded tiny GPT-2 (d=128, 2 layers,
2 heads, vocab 97, ctx 64, biases ~N(0, 0.02)) under each weight atom policy, the
prompt ids, the fp32 logits after every prompt position (Engine::step semantics,
gpt2.rs:227-332) and 16 greedy tokens (generate_greedy, gpt2.rs:367-388).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests.helpers import TINY, make_pack, oracle_engine, oracle_prefix_logits  # noqa: E402

POLICIES = ["auto", "q4auto", "core.f16", "f32"]


def case(policy: str):
    pk = make_pack(TINY, policy, 0, 0.02)
    eng = oracle_engine(pk)
    ids = ((np.arange(24) * 37 + 11) % TINY.vocab).astype(np.uint32)
    logits = oracle_prefix_logits(eng, ids)
    greedy = eng.generate_greedy(ids[:8], 16)
    return ids, logits, greedy


def main():
    for p in POLICIES:
        ids, logits, greedy = case(p)
        name = p.replace(".", "_")
        np.savez_compressed(os.path.join(HERE, f"tiny_{name}.npz"), ids=ids, logits=logits, greedy=greedy)
        print(p, logits.shape, greedy)


if __name__ == "__main__":
    main()
