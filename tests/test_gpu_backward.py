"""Backward kernels on the GPU (smelt_b200/csrc/backward.cu) through the C-ABI:
* each per-op kernel passes the reference's finite-difference self-check (gpu_backward.rs:
  915-1090, same seeds and tolerances) and matches the oracle's f64 ops on larger inputs;
* gpt2q_trunk_input_grad matches the oracle's trunk_input_grad (gpu_backward.rs:651-790) on the
  oracle's own f64 forward stash, and central differences of the f64 forward (bwparity.rs:690-735).
Tolerances: rel_max (the reference's metric, gpu_backward.rs:860-872) <= 2e-3 against the f64
oracle for the fp32 device computation; the self-checks use the reference's own bounds."""
import numpy as np
import pytest

from oracle import backward_oracle as B
from smelt_b200 import pack as P
from smelt_b200._ffi import Gpt2qError
from smelt_b200.backward import GpuBwdOps
from smelt_b200.gpu import Gpu

from .helpers import MINI, TINY, make_pack

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


@pytest.mark.parametrize("kernel", B.KERNELS)
def test_kernel_self_checks(kernel):
    mr, tol = B.selfcheck(GpuBwdOps(0), kernel)
    assert mr < tol, (kernel, mr, tol)


def test_ops_match_oracle_on_model_sizes():
    ops = GpuBwdOps(0)
    rng = np.random.default_rng(4)
    # lin_input_grad on a c_fc-shaped matrix (3072 x 768) and an odd one (100 x 1600)
    for rows, cols in ((3072, 768), (100, 1600), (5, 4)):
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        dy = rng.standard_normal(rows).astype(np.float32)
        got = ops.lin_input_grad(w, dy, rows, cols)
        ref = B.lin_input_grad(w.astype(np.float64), dy.astype(np.float64))
        assert B.rel_max(got, ref) < 2e-3, (rows, cols)
    # LayerNorm with accumulation into existing dg/db
    n = 768
    x = (rng.standard_normal(n) * 3 + 1).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    dy = rng.standard_normal(n).astype(np.float32)
    dg0 = rng.standard_normal(n).astype(np.float32)
    db0 = rng.standard_normal(n).astype(np.float32)
    dx, dg, db = ops.ln_backward(dy, x, g, np.zeros(n, np.float32), 1e-5, dg0, db0)
    rdx, rdg, rdb = B.ln_backward(dy[None].astype(np.float64), x[None].astype(np.float64), g.astype(np.float64), 1e-5)
    assert B.rel_max(dx, rdx[0]) < 2e-3
    assert np.allclose(dg, dg0 + rdg, rtol=1e-5, atol=1e-5) and np.allclose(db, db0 + rdb, rtol=1e-6, atol=1e-6)
    # GELU backward
    xp = (rng.standard_normal(5000) * 4).astype(np.float32)
    dyg = rng.standard_normal(5000).astype(np.float32)
    assert B.rel_max(ops.gelu_bwd(xp, dyg), B.gelu_bwd(xp.astype(np.float64), dyg.astype(np.float64))) < 2e-3
    # attention backward, 4 heads of 64, 70 positions, dk/dv accumulating onto non-zero inputs
    t, hd, stride = 70, 64, 256
    q, k, v, dya = (rng.standard_normal((t, stride)).astype(np.float32) for _ in range(4))
    dk0 = rng.standard_normal(t * stride).astype(np.float32)
    dv0 = rng.standard_normal(t * stride).astype(np.float32)
    dq, dk, dv = ops.attn_bwd_train(q, k, v, dya, t, hd, stride, dk0, dv0)
    rq, rk, rv = B.attn_bwd_train(*(a.astype(np.float64) for a in (q, k, v, dya)), hd)
    assert B.rel_max(dq, rq) < 2e-3
    assert B.rel_max(dk - dk0, rk) < 2e-3 and B.rel_max(dv - dv0, rv) < 2e-3


@pytest.mark.parametrize("meta,policy", [(TINY, "auto"), (TINY, "q4auto"), (TINY, "f32"), (MINI, "auto"),
                                         (MINI, "core.f16")])
def test_trunk_matches_oracle(meta, policy):
    pk = make_pack(meta, policy, 0, 0.02)
    W = B.weights64(pk)
    rng = np.random.default_rng(9)
    with Gpu(pk) as g:
        for n in (1, 7, 33, meta.n_ctx):
            ids = rng.integers(0, meta.vocab, n).astype(np.uint32)
            dl = B.sparse_dlogits(n, meta.vocab, seed=n)
            dx, lnf = g.trunk_input_grad(ids, dl)
            _, acts = B.forward_stash(W, meta, ids)
            ref = B.trunk_input_grad(W, meta, acts, dl.astype(np.float64))
            assert B.rel_max(dx, ref) < 2e-3, (n, B.rel_max(dx, ref))
            assert np.max(np.abs(lnf - acts["lnf_out"])) < 1e-3
            # a second call on the same handle gives the same result (deterministic kernels)
            if n == 33:
                dx2, _ = g.trunk_input_grad(ids, dl)
                assert np.array_equal(dx, dx2)


def test_trunk_matches_finite_differences():
    """The bwparity gate (bwparity.rs:690-735) with the device gradient: 32 wte coordinates."""
    pk = make_pack(TINY, "f32", 0, 0.02)
    W = B.weights64(pk)
    ids = np.array([11, 42, 11, 7, 96, 3, 42, 0], np.uint32)
    dl = B.sparse_dlogits(len(ids), TINY.vocab)
    with Gpu(pk) as g:
        dx, lnf = g.trunk_input_grad(ids, dl)
    rows = B.fd_embedding_check(W, TINY, ids, dl, dx, lnf)
    assert B.rel_max(rows[:, 0], rows[:, 1]) < 1e-2


def test_trunk_rejects_bad_arguments():
    pk = make_pack(TINY, "auto")
    with Gpu(pk) as g:
        ok = np.zeros((2, TINY.vocab), np.float32)
        with pytest.raises(Gpt2qError, match="vocab"):
            g.trunk_input_grad(np.array([1, TINY.vocab], np.uint32), ok)
        with pytest.raises(Gpt2qError, match="n out of range"):
            g.trunk_input_grad(np.zeros(TINY.n_ctx + 1, np.uint32), np.zeros((TINY.n_ctx + 1, TINY.vocab), np.float32))
        with pytest.raises(ValueError):
            g.trunk_input_grad(np.array([1, 2], np.uint32), np.zeros((3, TINY.vocab), np.float32))
        # the handle still works afterwards
        dx, _ = g.trunk_input_grad(np.array([1, 2], np.uint32), ok)
        assert np.all(dx == 0)


WIDE_VOCAB = P.Meta(n_embd=128, n_layer=2, n_head=2, n_ctx=64, vocab=9000)


@pytest.mark.parametrize("policy", ["auto", "q4auto", "f32"])
def test_trunk_head_on_tensor_cores(policy):
    """A vocabulary of >= 8192 rows with >= 16 positions takes the 3xTF32 tensor-core kernel for
    the head's transposed product (dh = dlogits . wte); the result matches the f64 oracle."""
    pk = make_pack(WIDE_VOCAB, policy, 0, 0.02)
    W = B.weights64(pk)
    rng = np.random.default_rng(21)
    with Gpu(pk) as g:
        for n in (16, 40, WIDE_VOCAB.n_ctx):
            ids = rng.integers(0, WIDE_VOCAB.vocab, n).astype(np.uint32)
            dl = (rng.standard_normal((n, WIDE_VOCAB.vocab)) * 0.01).astype(np.float32)  # dense dlogits
            dx, _ = g.trunk_input_grad(ids, dl)
            _, acts = B.forward_stash(W, WIDE_VOCAB, ids)
            ref = B.trunk_input_grad(W, WIDE_VOCAB, acts, dl.astype(np.float64))
            assert B.rel_max(dx, ref) < 2e-3, (n, B.rel_max(dx, ref))
