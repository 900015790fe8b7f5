"""ctypes front-end for the CPU oracle (oracle/oracle.cpp).

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product package (smelt_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)
_f64p = C.POINTER(C.c_double)
_u32p = C.POINTER(C.c_uint32)
_i64p = C.POINTER(C.c_int64)
_u64p = C.POINTER(C.c_uint64)

_lib = None


def build(out_dir: str | None = None, arch: str | None = None) -> str:
    """Compile the oracle with its Makefile; returns the .so path."""
    env = dict(os.environ)
    args = ["make", "-s", "-C", HERE]
    if out_dir:
        args.append(f"OUT={out_dir}")
    if arch:
        args.append(f"ARCH={arch}")
    subprocess.run(args, check=True, env=env)
    return os.path.join(out_dir or os.path.join(HERE, "_build"), "liboracle.so")


def _sig(lib):
    lib.orc_f32_to_f16.argtypes = [C.c_float]
    lib.orc_f32_to_f16.restype = C.c_uint16
    lib.orc_f16_to_f32.argtypes = [C.c_uint16]
    lib.orc_f16_to_f32.restype = C.c_float
    for fn in (lib.orc_q8_encode, lib.orc_q4_encode):
        fn.argtypes = [_f32p, C.c_size_t, _u8p]
        fn.restype = None
    for fn in (lib.orc_gemv_q8, lib.orc_gemv_q4, lib.orc_gemv_f16, lib.orc_gemv_f32):
        fn.argtypes = [_u8p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t]
        fn.restype = None
    lib.orc_pack_size.argtypes = [C.c_char_p, C.c_int, _i64p, C.c_char_p]
    lib.orc_pack_size.restype = C.c_size_t
    lib.orc_pack_tensor.argtypes = [C.c_char_p, C.c_int, _i64p, _f32p, C.c_char_p, _i64p,
                                    C.c_char_p, C.c_size_t, _u8p]
    lib.orc_pack_tensor.restype = C.c_int
    lib.orc_rng_new.argtypes = [C.c_uint64]
    lib.orc_rng_new.restype = C.c_uint64
    lib.orc_rng_normal_f32.argtypes = [_u64p, _f32p, C.c_size_t, C.c_double]
    lib.orc_rng_normal_f32.restype = None
    lib.orc_rng_below.argtypes = [_u64p, _u32p, C.c_size_t, C.c_uint64]
    lib.orc_rng_below.restype = None
    lib.orc_perf_atoms.argtypes = [_f64p, C.c_size_t]
    lib.orc_perf_atoms.restype = None
    lib.orc_engine_new.argtypes = [C.c_int] * 5 + [C.c_float, C.c_int]
    lib.orc_engine_new.restype = C.c_void_p
    lib.orc_engine_add.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_int, _i64p, _u8p,
                                   C.c_uint64]
    lib.orc_engine_add.restype = C.c_int
    lib.orc_engine_free.argtypes = [C.c_void_p]
    lib.orc_engine_free.restype = None
    lib.orc_kv_floats.argtypes = [C.c_void_p]
    lib.orc_kv_floats.restype = C.c_size_t
    lib.orc_engine_step.argtypes = [C.c_void_p, C.c_uint32, C.c_int, _f32p, _f32p]
    lib.orc_engine_step.restype = C.c_int
    lib.orc_engine_prefill.argtypes = [C.c_void_p, _u32p, C.c_int, C.c_int, _f32p, _f32p]
    lib.orc_engine_prefill.restype = C.c_int
    lib.orc_vec_f32.argtypes = [C.c_void_p, C.c_char_p, _f32p, C.c_uint64]
    lib.orc_vec_f32.restype = C.c_int
    lib.orc_vec_row.argtypes = [C.c_void_p, C.c_char_p, C.c_uint32, _f32p, C.c_uint64]
    lib.orc_vec_row.restype = C.c_int
    lib.orc_generate_greedy.argtypes = [C.c_void_p, _u32p, C.c_int, C.c_int, _u32p]
    lib.orc_generate_greedy.restype = C.c_int
    lib.orc_set_adapter.argtypes = [C.c_void_p, _f32p, _f32p, C.c_int]
    lib.orc_set_adapter.restype = C.c_int
    lib.orc_nll_per_token.argtypes = [C.c_void_p, _u32p, C.c_int]
    lib.orc_nll_per_token.restype = C.c_double
    lib.orc_argmax.argtypes = [_f32p, C.c_size_t]
    lib.orc_argmax.restype = C.c_uint32
    lib.orc_forward_f64.argtypes = [C.c_void_p, _u32p, C.c_int, _f64p]
    lib.orc_forward_f64.restype = C.c_int
    return lib


def lib(path: str | None = None):
    """Load (building first if needed) the oracle library."""
    global _lib
    if path is not None:
        return _sig(C.CDLL(path))
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = _sig(C.CDLL(LIB_PATH))
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


# ---------------------------------------------------------------- atoms
def f32_to_f16(x: float) -> int:
    return int(lib().orc_f32_to_f16(float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib().orc_f16_to_f32(int(h)))


def q8_encode(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib().orc_q8_encode(_p(x, _f32p), x.size, _p(out, _u8p))
    return out


def q4_encode(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * 18, dtype=np.uint8)
    lib().orc_q4_encode(_p(x, _f32p), x.size, _p(out, _u8p))
    return out


def gemv(atom: str, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    fn = {"core.i8.b32.f16scale": lib().orc_gemv_q8, "core.i4.b32.f16scale": lib().orc_gemv_q4,
          "core.f16": lib().orc_gemv_f16, "core.f32": lib().orc_gemv_f32}[atom]
    w = np.ascontiguousarray(w).view(np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    fn(_p(w, _u8p), _p(x, _f32p), _p(y, _f32p), rows, cols, 0, rows)
    return y


def pack_tensor(name: str, hf_shape, data: np.ndarray, policy: str):
    """Converter policy (pack.rs:47-84): returns (shape, atom, payload bytes)."""
    shp = np.asarray(hf_shape, dtype=np.int64)
    data = np.ascontiguousarray(data, dtype=np.float32)
    n = lib().orc_pack_size(name.encode(), len(shp), _p(shp, _i64p), policy.encode())
    out = np.empty(n, dtype=np.uint8)
    shape_out = np.zeros(len(shp), dtype=np.int64)
    atom = C.create_string_buffer(64)
    rc = lib().orc_pack_tensor(name.encode(), len(shp), _p(shp, _i64p), _p(data, _f32p),
                               policy.encode(), _p(shape_out, _i64p), atom, 64, _p(out, _u8p))
    if rc != 0:
        raise ValueError(f"orc_pack_tensor({name}) failed rc={rc}")
    return tuple(int(s) for s in shape_out), atom.value.decode(), out


# ---------------------------------------------------------------- RNG
class Rng:
    """xorshift64* (gpu_backward.rs:835-856) with the perf-lab Box-Muller normal."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(lib().orc_rng_new(seed))

    def normal_f32(self, n: int, std: float) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().orc_rng_normal_f32(C.byref(self.state), _p(out, _f32p), n, std)
        return out

    def below(self, n: int, bound: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint32)
        lib().orc_rng_below(C.byref(self.state), _p(out, _u32p), n, bound)
        return out


def perf_atoms(n_per_dist: int = 1 << 20) -> np.ndarray:
    out = np.zeros(40, dtype=np.float64)
    lib().orc_perf_atoms(_p(out, _f64p), n_per_dist)
    return out.reshape(20, 2)


# ---------------------------------------------------------------- engine
class Engine:
    """Oracle twin of the reference's CPU Engine (gpt2.rs:33-396)."""

    def __init__(self, meta: dict, tensors: dict, threads: int = 8):
        self.meta = dict(meta)
        self._l = lib()
        self.h = self._l.orc_engine_new(meta["n_embd"], meta["n_layer"], meta["n_head"],
                                        meta["n_ctx"], meta["vocab"], meta["ln_eps"], threads)
        self.shapes = {}
        for name, (shape, atom, data) in tensors.items():
            shp = np.asarray(shape, dtype=np.int64)
            data = np.ascontiguousarray(data).view(np.uint8)
            self._l.orc_engine_add(self.h, name.encode(), atom.encode(), len(shp), _p(shp, _i64p),
                                   _p(data, _u8p), data.size)
            self.shapes[name] = tuple(shape)

    def __del__(self):
        if getattr(self, "h", None):
            self._l.orc_engine_free(self.h)
            self.h = None

    def empty_kv(self) -> np.ndarray:
        return np.zeros(self._l.orc_kv_floats(self.h), dtype=np.float32)

    def step(self, tok: int, pos: int, kv: np.ndarray) -> np.ndarray:
        logits = np.empty(self.meta["vocab"], dtype=np.float32)
        rc = self._l.orc_engine_step(self.h, int(tok), int(pos), _p(kv, _f32p), _p(logits, _f32p))
        if rc != 0:
            raise ValueError(f"orc_engine_step rc={rc}")
        return logits

    def prefill(self, ids, kv: np.ndarray, pos0: int = 0) -> np.ndarray:
        """len(ids) consecutive `step` calls at positions pos0.. (the prompt loop, gpt2.rs:373-381),
        computed over all positions at once with bit-identical results: fills kv and returns the
        logits of the last position."""
        p = np.ascontiguousarray(ids, dtype=np.uint32)
        logits = np.empty(self.meta["vocab"], dtype=np.float32)
        rc = self._l.orc_engine_prefill(self.h, _p(p, _u32p), p.size, int(pos0), _p(kv, _f32p), _p(logits, _f32p))
        if rc != 0:
            raise ValueError(f"orc_engine_prefill rc={rc}")
        return logits

    def vec_f32(self, name: str) -> np.ndarray:
        n = int(np.prod(self.shapes[name]))
        out = np.empty(n, dtype=np.float32)
        if self._l.orc_vec_f32(self.h, name.encode(), _p(out, _f32p), n) != 0:
            raise KeyError(name)
        return out

    def generate_greedy(self, prompt, steps: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(steps, dtype=np.uint32)
        n = self._l.orc_generate_greedy(self.h, _p(p, _u32p), p.size, steps, _p(out, _u32p))
        return out[:n]

    def set_adapter(self, a=None, b=None):
        """Post-ln_f adapter h += B (A h) (gpu.rs:188-194, cu/gpt2.cu:196-215); None clears."""
        if a is None:
            self._l.orc_set_adapter(self.h, None, None, 0)
            return
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        r = a.shape[0]
        assert a.shape == (r, self.meta["n_embd"]) and b.shape == (self.meta["n_embd"], r)
        self._l.orc_set_adapter(self.h, _p(a, _f32p), _p(b, _f32p), r)

    def nll_per_token(self, ids) -> float:
        p = np.ascontiguousarray(ids, dtype=np.uint32)
        return float(self._l.orc_nll_per_token(self.h, _p(p, _u32p), p.size))

    def forward_f64(self, ids) -> np.ndarray:
        p = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.empty((p.size, self.meta["vocab"]), dtype=np.float64)
        self._l.orc_forward_f64(self.h, _p(p, _u32p), p.size, _p(out, _f64p))
        return out


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().orc_argmax(_p(v, _f32p), v.size))
