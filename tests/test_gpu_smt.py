"""A handle made straight from an SMT file (gpt2q_create_from_smt: Engine::load + Gpu::new,
gpt2.rs:43-89, gpu.rs:75-157) computes exactly what a handle made from the same pack in
memory computes, and matches the oracle; a corrupted file is refused before any upload."""
import numpy as np
import pytest

from smelt_b200 import smt
from smelt_b200._ffi import Gpt2qError
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack, oracle_engine, oracle_prefix_logits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


@pytest.mark.parametrize("meta,policy", [(TINY, "auto"), (TINY, "q4auto"), (MINI, "auto"), (MINI, "f32")])
def test_smt_handle_is_bit_identical_to_pack_handle(tmp_path, meta, policy):
    pk = make_pack(meta, policy, 0, 0.02)
    path = str(tmp_path / "m.smt")
    smt.write_smt(path, pk)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, meta.vocab, n).astype(np.uint32) for n in (1, 9, 23)]
    with Gpu(pk, max_seqs=3) as a, Gpu.from_smt(path, max_seqs=3) as b:
        assert b.meta == pk.meta
        na, la = a.prefill(prompts, want_logits=True)
        nb, lb = b.prefill(prompts, want_logits=True)
        assert np.array_equal(la, lb) and np.array_equal(na, nb)
        ta = a.decode_steps(6, 3)
        tb = b.decode_steps(6, 3)
        assert np.array_equal(ta, tb)
        for name in ("h.0.attn.c_attn.weight", "wte.weight"):
            numel = pk.tensors[name].numel
            assert np.array_equal(a.dequant(name, numel), b.dequant(name, numel))
    eng = oracle_engine(pk)
    ref = oracle_prefix_logits(eng, prompts[1])[-1]
    assert np.max(np.abs(lb[1] - ref)) <= 2e-2


def test_corrupted_smt_is_refused(tmp_path):
    pk = make_pack(TINY, "auto")
    path = str(tmp_path / "m.smt")
    smt.write_smt(path, pk)
    buf = bytearray(open(path, "rb").read())
    buf[len(buf) // 2] ^= 0x40
    bad = str(tmp_path / "bad.smt")
    open(bad, "wb").write(bytes(buf))
    with pytest.raises(Gpt2qError, match="merkle"):
        Gpu.from_smt(bad)
    with Gpu.from_smt(path, verify=True) as g:
        assert g.prefill([np.array([1, 2, 3], np.uint32)]).shape == (1,)
