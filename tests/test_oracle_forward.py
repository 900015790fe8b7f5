"""The oracle forward against two independent forwards.

1. the reference's own float64 full-sequence forward (bwparity.rs:215-305),
   restated as orc_forward_f64;
2. Hugging Face transformers' GPT2LMHeadModel in float64 with the same
   dequantised weights (the architecture the reference packs were converted from).
"""
import numpy as np
import pytest
import torch

from smelt_b200 import pack as P

from .helpers import MINI, TINY, make_pack, oracle_engine, oracle_prefix_logits


@pytest.mark.parametrize("policy", ["auto", "q4auto", "f32"])
def test_step_matches_f64_forward(policy):
    pk = make_pack(TINY, policy, 0, 0.02)
    eng = oracle_engine(pk)
    ids = np.arange(20) * 7 % TINY.vocab
    a = oracle_prefix_logits(eng, ids)
    b = eng.forward_f64(ids)
    assert np.abs(a - b).max() < 1e-4


def hf_model(pk: P.Pack):
    from transformers import GPT2Config, GPT2LMHeadModel
    m = pk.meta
    cfg = GPT2Config(n_embd=m.n_embd, n_layer=m.n_layer, n_head=m.n_head, vocab_size=m.vocab,
                     n_positions=m.n_ctx, layer_norm_epsilon=m.ln_eps, activation_function="gelu_new",
                     attn_implementation="eager")
    model = GPT2LMHeadModel(cfg).double().eval()
    sd = {}
    for name, t in pk.tensors.items():
        w = pk.dequant(name).astype(np.float64)
        if len(t.shape) == 2 and name.endswith(P.CONV1D_SUFFIXES):
            w = w.T  # back to HF Conv1D [in, out]
        sd["transformer." + name] = torch.from_numpy(np.ascontiguousarray(w))
    sd["lm_head.weight"] = sd["transformer.wte.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected
    return model


@pytest.mark.parametrize("meta", [TINY, MINI])
def test_step_matches_transformers_float64(meta):
    pk = make_pack(meta, "auto", 0, 0.02)
    eng = oracle_engine(pk)
    ids = (np.arange(24) * 13 + 5) % meta.vocab
    ours = oracle_prefix_logits(eng, ids)
    with torch.no_grad():
        ref = hf_model(pk)(torch.from_numpy(ids.astype(np.int64))[None]).logits[0].numpy()
    assert np.abs(ours - ref).max() < 1e-4
    assert np.array_equal(ours.argmax(-1), ref.argmax(-1))


def test_greedy_and_nll_consistent():
    pk = make_pack(TINY, "auto")
    eng = oracle_engine(pk)
    prompt = np.array([3, 14, 15, 92, 65], np.uint32)
    g1 = eng.generate_greedy(prompt, 12)
    g2 = eng.generate_greedy(prompt, 12)
    assert np.array_equal(g1, g2) and g1.size == 12
    # first generated token is the argmax of the last prompt position (gpt2.rs:379-381)
    logits = oracle_prefix_logits(eng, prompt)
    from oracle import oracle as O
    assert g1[0] == O.argmax(logits[-1])
    nll = eng.nll_per_token(np.concatenate([prompt, g1]))
    assert np.isfinite(nll) and nll > 0


def test_greedy_stops_at_context():
    pk = make_pack(TINY, "auto")
    eng = oracle_engine(pk)
    prompt = np.arange(60, dtype=np.uint32) % TINY.vocab
    out = eng.generate_greedy(prompt, 10)
    # positions 59..63 produce 5 tokens before pos > n_ctx-1 stops generation
    assert out.size == TINY.n_ctx - prompt.size + 1


def test_argmax_ties_pick_last():
    from oracle import oracle as O
    v = np.array([1.0, 5.0, 2.0, 5.0, 5.0, -1.0], np.float32)
    assert O.argmax(v) == 4
    assert O.argmax(np.array([0.0, -0.0], np.float32)) == 0  # +0 > -0 in total order
