"""gpt2q_argmax_noalloc: the greedy argmax for callers that cannot allocate device memory.

Loops that must never stall the device on cudaMalloc/cudaFree, or code running under
another framework's memory pool, cannot let the library allocate scratch at call time. This entry point keeps its scratch
in a fixed array inside the library; the caller passes device logits in and gets device
token ids out. The test checks it against the tokens the regular decode path returns,
on two calls in a row (the shared scratch must come back clean after each call).
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from smelt_b200 import _ffi
from smelt_b200.gpu import Gpu

from .helpers import MINI, make_pack

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    from smelt_b200 import build
    build.build()


def _call(lib, d_logits, vocab, ld, n_rows, d_next, stream):
    return lib.gpt2q_argmax_noalloc(C.c_void_p(d_logits.data_ptr()), vocab, ld, n_rows,
                                    C.c_void_p(d_next.data_ptr()), C.c_void_p(stream.cuda_stream))


def test_argmax_noalloc_matches_decode_path():
    import torch

    pk = make_pack(MINI, "auto", 0, 0.02)
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, MINI.vocab, n).astype(np.uint32) for n in (5, 17, 40)]
    with Gpu(pk, max_seqs=len(prompts)) as g:
        nxt0, lg0 = g.prefill(prompts, want_logits=True)
        nxt1, lg1 = g.decode(nxt0, [p.size for p in prompts], want_logits=True)
    lib = _ffi.load()
    stream = torch.cuda.Stream()
    V = MINI.vocab
    for lg, ref in ((lg0, nxt0), (lg1, nxt1)):  # two calls in a row share the scratch
        d_logits = torch.from_numpy(np.ascontiguousarray(lg)).cuda()
        d_next = torch.full((lg.shape[0],), -1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        assert _call(lib, d_logits, V, V, lg.shape[0], d_next, stream) == 0
        stream.synchronize()
        got = d_next.cpu().numpy().view(np.uint32)
        assert np.array_equal(got, ref), (got, ref)


def test_argmax_noalloc_ties_row_stride_and_limit():
    import torch

    lib = _ffi.load()
    stream = torch.cuda.Stream()
    V, ld, n = 5000, 5004, 7
    rng = np.random.default_rng(4)
    lg = rng.standard_normal((n, ld)).astype(np.float32)
    lg[:, V:] = 1e30  # padding past vocab must be ignored
    lg[2, [10, 20, 4999]] = 9.0  # ties: the LAST maximal index wins (gpt2.rs:390-396)
    lg[5, :V] = 0.0
    lg[5, 3] = -0.0
    d_logits = torch.from_numpy(lg).cuda()
    d_next = torch.zeros(n, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    assert _call(lib, d_logits, V, ld, n, d_next, stream) == 0
    stream.synchronize()
    got = d_next.cpu().numpy().view(np.uint32)
    ref = np.array([O.argmax(lg[i, :V]) for i in range(n)], np.uint32)
    assert np.array_equal(got, ref) and got[2] == 4999
    big = torch.zeros((_ffi_max() + 1, 8), dtype=torch.float32, device="cuda")
    out = torch.zeros(_ffi_max() + 1, dtype=torch.int32, device="cuda")
    assert _call(lib, big, 8, 8, _ffi_max() + 1, out, stream) == -1
    assert b"exceeds the maximum" in lib.gpt2q_last_error(None)


@pytest.mark.parametrize("n_rows,vocab", [(None, 33), (3, 3 * 4096 + 17)])
def test_argmax_noalloc_full_array_and_wide_vocabulary(n_rows, vocab):
    """Exactly GPT2Q_NOALLOC_MAX_ROWS rows (the whole scratch array), and a vocabulary that
    spans several argmax blocks per row; each checked twice in a row against the oracle."""
    import torch

    lib = _ffi.load()
    stream = torch.cuda.Stream()
    n = n_rows or _ffi_max()
    rng = np.random.default_rng(n + vocab)
    for rep in range(2):
        lg = rng.standard_normal((n, vocab)).astype(np.float32)
        lg[::7, vocab // 2] = 50.0 + rep  # a clear maximum in the middle of some rows
        d_logits = torch.from_numpy(lg).cuda()
        d_next = torch.full((n,), -1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        assert _call(lib, d_logits, vocab, vocab, n, d_next, stream) == 0
        stream.synchronize()
        got = d_next.cpu().numpy().view(np.uint32)
        ref = np.array([O.argmax(lg[i]) for i in range(n)], np.uint32)
        assert np.array_equal(got, ref)


def _ffi_max() -> int:
    import os

    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "gpt2q.h")).read()
    for line in hdr.splitlines():
        if line.startswith("#define GPT2Q_NOALLOC_MAX_ROWS"):
            return int(line.split()[2])
    raise AssertionError("GPT2Q_NOALLOC_MAX_ROWS not declared")
