"""The oracle still reproduces the committed golden fixtures (regression pin)."""
import os

import numpy as np
import pytest

from .golden.make_golden import POLICIES, case

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("policy", POLICIES)
def test_oracle_reproduces_golden(policy):
    g = np.load(os.path.join(HERE, "golden", f"tiny_{policy.replace('.', '_')}.npz"))
    ids, logits, greedy = case(policy)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(logits.view(np.uint32), g["logits"].view(np.uint32))
    assert np.array_equal(greedy, g["greedy"])
