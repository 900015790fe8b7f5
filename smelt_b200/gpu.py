"""Python mirror of model-lab's CUDA executor API on top of libgpt2q.so.

`Gpu` keeps the shape of LukasParke/smelt's `Gpu` (experiments/model-lab/src/
gpu.rs:51-379): construct from a weight pack, `step(tok, pos)` returns the fp32
logits of one position, `clear_kv()` resets the cache, `launches` counts kernels.
The reference panics on CUDA errors; here every failure raises Gpt2qError with
the library's message. Batched prefill/decode/greedy generation and device-side
multi-step decode are the additions this B200 build is for.
"""
from __future__ import annotations

import ctypes as C
import json

import numpy as np

from . import _ffi
from .pack import Meta, Pack


def _descs(pack: Pack):
    arr = (_ffi.TensorDesc * len(pack.tensors))()
    keep = []
    for i, (name, t) in enumerate(pack.tensors.items()):
        data = np.ascontiguousarray(t.data)
        keep.append(data)
        nb, ab = name.encode(), t.atom.encode()
        keep += [nb, ab]
        arr[i].name = nb
        arr[i].atom = ab
        arr[i].ndim = len(t.shape)
        for k, s in enumerate(t.shape):
            arr[i].shape[k] = s
        arr[i].data = data.ctypes.data
        arr[i].len = data.nbytes
    return arr, keep


class Gpu:
    def __init__(self, pack: Pack, device: int = 0, max_seqs: int = 1, max_tokens: int = 0,
                 tp_size: int = 1, tp_rank: int = 0, nccl_id: bytes | None = None):
        self._lib = _ffi.load()
        self.meta = pack.meta
        cfg = _ffi.Config(pack.meta.n_embd, pack.meta.n_layer, pack.meta.n_head, pack.meta.n_ctx,
                          pack.meta.vocab, pack.meta.ln_eps, max_seqs, max_tokens)
        descs, keep = _descs(pack)
        h = C.c_void_p()
        if tp_size > 1:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("tensor-parallel Gpu needs the 128-byte NCCL unique id")
            idbuf = C.create_string_buffer(bytes(nccl_id), 128)
            rc = self._lib.gpt2q_create_tp(C.byref(cfg), descs, len(pack.tensors), device, tp_size, tp_rank,
                                           idbuf, C.byref(h))
        else:
            rc = self._lib.gpt2q_create(C.byref(cfg), descs, len(pack.tensors), device, C.byref(h))
        del keep
        _ffi.check(self._lib, None, rc)
        self.h = h
        self.max_seqs = max_seqs
        self.device = device

    @classmethod
    def from_smt(cls, path: str, device: int = 0, max_seqs: int = 1, max_tokens: int = 0,
                 verify: bool = True) -> "Gpu":
        """Engine::load + Gpu::new (gpt2.rs:43-89, gpu.rs:75-157) straight from an SMT file:
        the library maps the file, verifies the merkle content_id and every tensor digest
        (unless verify=False) and uploads the tensors; any mismatch raises Gpt2qError."""
        from .smt import inspect
        arch = inspect(path, verify=False)["arch"]
        self = cls.__new__(cls)
        self._lib = _ffi.load()
        self.meta = Meta(arch["n_embd"], arch["n_layer"], arch["n_head"], arch["n_ctx"], arch["vocab_size"])
        h = C.c_void_p()
        rc = self._lib.gpt2q_create_from_smt(str(path).encode(), device, max_seqs, max_tokens, 1 if verify else 0,
                                             C.byref(h))
        _ffi.check(self._lib, None, rc)
        self.h = h
        self.max_seqs = max_seqs
        self.device = device
        return self

    # ---- lifetime ----
    def close(self):
        if getattr(self, "h", None):
            self._lib.gpt2q_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc: int):
        _ffi.check(self._lib, self.h, rc)

    # ---- reference-shaped API (gpu.rs) ----
    def step(self, tok: int, pos: int) -> np.ndarray:
        """Gpu::step (gpu.rs:212): one token of sequence slot 0 -> vocab logits."""
        out = np.empty(self.meta.vocab, dtype=np.float32)
        self._check(self._lib.gpt2q_step(self.h, int(tok), int(pos), out.ctypes.data_as(_ffi._f32p)))
        return out

    def clear_kv(self, slots=None):
        """Gpu::clear_kv (gpu.rs:203)."""
        if slots is None:
            self._check(self._lib.gpt2q_reset_kv(self.h, None, 0))
        else:
            s = np.ascontiguousarray(slots, dtype=np.int32)
            self._check(self._lib.gpt2q_reset_kv(self.h, s.ctypes.data_as(_ffi._i32p), s.size))

    @property
    def launches(self) -> int:
        return int(self._lib.gpt2q_launches(self.h))

    # ---- batched API ----
    def decode(self, tok, pos, slots=None, want_logits: bool = False):
        tok = np.ascontiguousarray(tok, dtype=np.uint32)
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        n = tok.size
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        nxt = np.empty(n, dtype=np.uint32)
        lg = np.empty((n, self.meta.vocab), dtype=np.float32) if want_logits else None
        self._check(self._lib.gpt2q_decode(
            self.h, tok.ctypes.data, pos.ctypes.data, None if sl is None else sl.ctypes.data, n,
            None if lg is None else lg.ctypes.data, nxt.ctypes.data))
        return (nxt, lg) if want_logits else nxt

    @staticmethod
    def _flatten(prompts):
        prompts = [np.ascontiguousarray(p, dtype=np.uint32) for p in prompts]
        offs = np.zeros(len(prompts) + 1, dtype=np.int32)
        offs[1:] = np.cumsum([p.size for p in prompts])
        toks = np.concatenate(prompts) if prompts else np.zeros(0, np.uint32)
        return np.ascontiguousarray(toks, dtype=np.uint32), offs

    def prefill(self, prompts, slots=None, want_logits: bool = False):
        toks, offs = self._flatten(prompts)
        n = len(prompts)
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        nxt = np.empty(n, dtype=np.uint32)
        lg = np.empty((n, self.meta.vocab), dtype=np.float32) if want_logits else None
        self._check(self._lib.gpt2q_prefill(
            self.h, toks.ctypes.data_as(_ffi._u32p), offs.ctypes.data_as(_ffi._i32p),
            None if sl is None else sl.ctypes.data_as(_ffi._i32p), n,
            None if lg is None else lg.ctypes.data_as(_ffi._f32p), nxt.ctypes.data_as(_ffi._u32p)))
        return (nxt, lg) if want_logits else nxt

    def decode_steps(self, steps: int, n_seq: int, want_tokens: bool = True):
        out = np.empty((steps, n_seq), dtype=np.uint32) if want_tokens else None
        self._check(self._lib.gpt2q_decode_steps(
            self.h, int(steps), None if out is None else out.ctypes.data_as(_ffi._u32p)))
        return out

    def generate_greedy(self, prompts, steps: int) -> np.ndarray:
        """generate_greedy (gpt2.rs:367-388) for every prompt; returns [n_seq, steps]."""
        toks, offs = self._flatten(prompts)
        out = np.empty((len(prompts), steps), dtype=np.uint32)
        self._check(self._lib.gpt2q_generate_greedy(
            self.h, toks.ctypes.data_as(_ffi._u32p), offs.ctypes.data_as(_ffi._i32p), len(prompts), int(steps),
            out.ctypes.data_as(_ffi._u32p)))
        return out

    def set_adapter(self, a, b):
        """Publish a post-ln_f adapter h += B (A h) (Gpu::set_adapter, gpu.rs:188-194):
        a [r, d], b [d, r] float32; later steps use it."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        r = a.shape[0]
        if a.shape != (r, self.meta.n_embd) or b.shape != (self.meta.n_embd, r):
            raise ValueError("adapter shapes must be a [r, d] and b [d, r]")
        self._check(self._lib.gpt2q_set_adapter(self.h, a.ctypes.data_as(_ffi._f32p), b.ctypes.data_as(_ffi._f32p),
                                                int(r)))

    def clear_adapter(self):
        self._check(self._lib.gpt2q_clear_adapter(self.h))

    def nll(self, ids, slot: int = 0) -> float:
        """Teacher-forced NLL per token (nll_per_token, gpt2.rs:347-364), computed on the
        device; overwrites the KV cache of `slot`."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = C.c_double(0.0)
        self._check(self._lib.gpt2q_nll(self.h, ids.ctypes.data_as(_ffi._u32p), int(ids.size), int(slot),
                                        C.byref(out)))
        return float(out.value)

    def trunk_input_grad(self, ids, dlogits):
        """(dx [n][n_embd], lnf_out [n][n_embd]): the trunk input gradient of trunk_input_grad
        (gpu_backward.rs:651-790) for dlogits [n][vocab], forward and backward on the device."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        n = ids.size
        dl = np.ascontiguousarray(dlogits, dtype=np.float32)
        if dl.shape != (n, self.meta.vocab):
            raise ValueError(f"dlogits must be [{n}][{self.meta.vocab}]")
        dx = np.empty((n, self.meta.n_embd), np.float32)
        lnf = np.empty((n, self.meta.n_embd), np.float32)
        self._check(self._lib.gpt2q_trunk_input_grad(self.h, ids.ctypes.data_as(_ffi._u32p), n,
                                                     dl.ctypes.data_as(_ffi._f32p), dx.ctypes.data_as(_ffi._f32p),
                                                     lnf.ctypes.data_as(_ffi._f32p)))
        return dx, lnf

    def dequant(self, name: str, numel: int) -> np.ndarray:
        out = np.empty(numel, dtype=np.float32)
        self._check(self._lib.gpt2q_dequant(self.h, name.encode(), out.ctypes.data_as(_ffi._f32p), numel))
        return out

    # ---- plumbing ----
    def set_stream(self, stream_handle: int | None):
        self._check(self._lib.gpt2q_set_stream(self.h, C.c_void_p(stream_handle or 0)))

    def sync(self):
        self._check(self._lib.gpt2q_sync(self.h))

    def profile(self, enable: bool):
        self._check(self._lib.gpt2q_profile(self.h, 1 if enable else 0))

    def profile_kernels(self, reps: int = 20) -> dict:
        """Steady-state per-launch time of every kernel type of one decode step."""
        buf = C.create_string_buffer(1 << 16)
        self._check(self._lib.gpt2q_profile_kernels(self.h, int(reps), buf, len(buf)))
        return json.loads(buf.value.decode())

    def info(self) -> dict:
        """Execution paths of this handle (persistent single-sequence decode, tensor cores)."""
        buf = C.create_string_buffer(1 << 20)
        self._check(self._lib.gpt2q_info(self.h, buf, len(buf)))
        return json.loads(buf.value.decode())

    def profile_read(self) -> dict:
        buf = C.create_string_buffer(1 << 16)
        self._check(self._lib.gpt2q_profile_read(self.h, buf, len(buf)))
        return json.loads(buf.value.decode())
