"""The oracle's restatement of the trunk backward (oracle/backward_oracle.py) on its own: its four
ops pass the reference's finite-difference self-checks (gpu_backward.rs:915-1090), and the
composed trunk_input_grad (gpu_backward.rs:651-790) agrees with central differences of the f64
forward (bwparity.rs:690-735) on small models. CPU only."""
import numpy as np
import pytest

from oracle import backward_oracle as B

from .helpers import MINI, TINY, make_pack


@pytest.mark.parametrize("kernel", B.KERNELS)
def test_mirror_ops_pass_reference_self_checks(kernel):
    mr, tol = B.selfcheck(B.MirrorOps(), kernel)
    assert mr < tol, (kernel, mr, tol)


def test_rng_matches_reference_definition():
    """xorshift64* with seed ^ 0x9E3779B97F4A7C15 (gpu_backward.rs:838-856): first outputs by hand."""
    r = B.Rng(0)
    x = 0x9E3779B97F4A7C15
    x ^= x >> 12
    x ^= (x << 25) & B.M64
    x ^= x >> 27
    assert r.next_u64() == (x * 0x2545F4914F6CDD1D) & B.M64
    r = B.Rng(7)
    vals = [r.f32() for _ in range(1000)]
    assert all(-1.0 <= v < 1.0 for v in vals) and all(v.dtype == np.float32 for v in vals)


@pytest.mark.parametrize("meta,policy", [(TINY, "f32"), (TINY, "auto"), (MINI, "q4auto")])
def test_trunk_composition_matches_finite_differences(meta, policy):
    pk = make_pack(meta, policy, 0, 0.02)
    W = B.weights64(pk)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, meta.vocab, 6).astype(np.uint32)
    ids[3] = ids[0]  # a repeated token: the input path sums over its positions
    dl = B.sparse_dlogits(len(ids), meta.vocab)
    _, acts = B.forward_stash(W, meta, ids)
    dx = B.trunk_input_grad(W, meta, acts, dl.astype(np.float64))
    rows = B.fd_embedding_check(W, meta, ids, dl, dx, acts["lnf_out"], n_coords=16)
    assert B.rel_max(rows[:, 0], rows[:, 1]) < 1e-3


@pytest.mark.parametrize("policy", ["f32", "auto"])
def test_f64_stash_forward_agrees_with_the_cpp_oracle(policy):
    """The backward oracle's f64 forward (bwparity.rs forward_stash) and the C++ restatement of
    Engine::step give the same logits on the same dequantised weights (to f32 rounding)."""
    from .helpers import oracle_engine, oracle_prefix_logits

    pk = make_pack(TINY, policy, 0, 0.02)
    ids = np.array([3, 14, 15, 92, 65, 35, 89], np.uint32)
    lg64, _ = B.forward_stash(B.weights64(pk), TINY, ids)
    lg32 = oracle_prefix_logits(oracle_engine(pk), ids)
    assert np.max(np.abs(lg64 - lg32)) < 1e-4


def _rust_e(v: float, prec: int) -> str:
    """Rust's `{:.Ne}` formatting (no exponent padding, no '+')."""
    mant, exp = f"{v:.{prec}e}".split("e")
    return f"{mant}e{int(exp)}"


def test_mirror32_reproduces_the_reference_kcheck_log():
    """The f32 restatement of MirrorOps run through the restated self-check harness prints the
    reference's own KCHECK lines for its CPU mirror, digit for digit
    (docs/experiments/results/bwparity.log:6-9, copied to tests/golden/bwparity_kcheck_ref.txt).
    This pins the Rng, the finite-difference harness and rel_max, and the mirror arithmetic."""
    import os

    samples = {"k_lin_input_grad": 24, "k_ln_backward": 192, "k_gelu_bwd": 32, "k_attn_bwd_train": 120}
    lines = []
    for k in B.KERNELS:
        mr, tol = B.selfcheck(B.MirrorOps32(), k)
        lines.append(f"KCHECK {k} [cpu-mirror] samples={samples[k]} max_rel={_rust_e(mr, 3)} "
                     f"tol={_rust_e(tol, 0)} {'PASS' if mr < tol else 'FAIL'}")
    ref = open(os.path.join(os.path.dirname(__file__), "golden", "bwparity_kcheck_ref.txt")).read().splitlines()
    assert lines == ref


def test_per_op_entry_points_refuse_bad_arguments_before_any_device_call():
    """The per-op backward C-ABI (gpt2q_bwd_*) checks its arguments on the host and returns
    EARG with a message before it opens a device, so these calls need no GPU."""
    import ctypes as C

    from smelt_b200 import _ffi, build

    build.build()
    lib = _ffi.load()
    f = np.zeros(64, np.float32)
    p = f.ctypes.data_as(C.POINTER(C.c_float))
    null = C.POINTER(C.c_float)()
    cases = [
        (lib.gpt2q_bwd_lin_input_grad, (0, p, p, 4, 6, p), "cols % 4"),      # cols not a multiple of 4
        (lib.gpt2q_bwd_lin_input_grad, (0, p, null, 4, 8, p), "null"),
        (lib.gpt2q_bwd_lin_input_grad, (0, p, p, 0, 8, p), "rows/cols"),
        (lib.gpt2q_bwd_ln_backward, (0, p, p, p, p, 1e-5, 0, p, p, p), "null"),
        (lib.gpt2q_bwd_gelu, (0, p, p, -1, p), "null"),
        (lib.gpt2q_bwd_attn_train, (0, p, p, p, p, 4, 64, 96, p, p, p), "stride"),   # stride % hd != 0
        (lib.gpt2q_bwd_attn_train, (0, p, p, p, p, 1025, 64, 64, p, p, p), "t <= 1024"),
        (lib.gpt2q_bwd_attn_train, (0, p, p, p, p, 4, 256, 256, p, p, p), "hd <= 128"),
    ]
    for fn, args, words in cases:
        assert fn(*args) == -1, (fn.__name__, args)
        assert words in lib.gpt2q_last_error(None).decode(), (fn.__name__, words)
    assert lib.gpt2q_trunk_input_grad(None, None, 1, None, None, None) == -1
