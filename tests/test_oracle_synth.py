"""The oracle-side model generator (oracle/synth.py, used by the benchmark's reference arm so that
it never loads the product library) produces exactly the product generator's weights and token
ids: same Rng stream (gpu_backward.rs:835-856), same converter (pack.rs:47-84)."""
import numpy as np
import pytest

from oracle import synth as OS
from smelt_b200 import pack as P
from smelt_b200 import synth

from .helpers import MINI, TINY, make_pack


@pytest.mark.parametrize("bias_std", [0.0, 0.02])
@pytest.mark.parametrize("policy", ["auto", "q4auto", "core.f16", "f32"])
@pytest.mark.parametrize("meta", [TINY, MINI], ids=["tiny", "mini"])
def test_oracle_model_equals_product_pack(meta, policy, bias_std):
    pk = make_pack(meta, policy, 0, bias_std)
    ot = OS.synthetic_tensors(meta.as_dict(), policy, 0, bias_std=bias_std)
    assert list(ot) == list(pk.tensors)
    for name, t in pk.tensors.items():
        shape, atom, data = ot[name]
        assert shape == t.shape and atom == t.atom and np.array_equal(data, t.data), name


def test_streamed_pack_equals_whole_conversion():
    a = synth.synthetic_pack(MINI, "auto", seed=3, bias_std=0.02)
    b = P.from_hf(MINI, synth.hf_weights(MINI, seed=3, bias_std=0.02), "auto")
    assert list(a.tensors) == list(b.tensors)
    for n in a.tensors:
        assert np.array_equal(a.tensors[n].data, b.tensors[n].data), n


def test_token_ids_and_lengths_match():
    assert np.array_equal(OS.prompt_ids(5000, 50257, seed=1), synth.prompt_ids(5000, 50257, seed=1))
    assert np.array_equal(OS.ragged_lengths(256, 16, 512, seed=2), synth.ragged_lengths(256, 16, 512, seed=2))


def test_model_configs_agree():
    for name in ("small", "medium", "xl"):
        assert OS.MODELS[name] == P.CONFIGS[name].as_dict()
    assert OS.hf_shapes(MINI.as_dict()) == P.hf_shapes(MINI)
