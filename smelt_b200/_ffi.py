"""ctypes binding of libgpt2q.so (include/gpt2q.h).

There is no fallback: if the library is missing the import of the GPU entry
points fails loudly. Build it with ``python -m smelt_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libgpt2q.so")

GPT2Q_OK = 0
ERRORS = {-1: "EARG", -2: "EOOM", -3: "ECUDA", -4: "ENCCL", -5: "ETIMEOUT", -6: "EUNSUP"}

# Every symbol declared in include/gpt2q.h.
EXPORTS = [
    "gpt2q_create", "gpt2q_create_tp", "gpt2q_destroy", "gpt2q_last_error", "gpt2q_reset_kv",
    "gpt2q_step", "gpt2q_decode", "gpt2q_prefill", "gpt2q_decode_steps", "gpt2q_generate_greedy",
    "gpt2q_dequant", "gpt2q_launches", "gpt2q_set_stream", "gpt2q_sync", "gpt2q_profile",
    "gpt2q_profile_read", "gpt2q_profile_kernels", "gpt2q_info", "gpt2q_argmax_noalloc", "gpt2q_rng_new", "gpt2q_rng_normal_f32", "gpt2q_rng_below",
    "gpt2q_quantize_q8", "gpt2q_quantize_q4", "gpt2q_nll",
    "gpt2q_set_adapter", "gpt2q_clear_adapter",
    "gpt2q_create_from_smt", "gpt2q_smt_inspect", "gpt2q_blake3",
    "gpt2q_trunk_input_grad", "gpt2q_bwd_lin_input_grad", "gpt2q_bwd_ln_backward", "gpt2q_bwd_gelu",
    "gpt2q_bwd_attn_train",
]


class Config(C.Structure):
    _fields_ = [("n_embd", C.c_int32), ("n_layer", C.c_int32), ("n_head", C.c_int32),
                ("n_ctx", C.c_int32), ("vocab", C.c_int32), ("ln_eps", C.c_float),
                ("max_seqs", C.c_int32), ("max_tokens", C.c_int32)]


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("atom", C.c_char_p), ("ndim", C.c_int32),
                ("shape", C.c_int64 * 2), ("data", C.c_void_p), ("len", C.c_uint64)]


class Gpt2qError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"gpt2q error {code} ({ERRORS.get(code, '?')}): {msg}")
        self.code = code


_lib = None

_u32p = C.POINTER(C.c_uint32)
_i32p = C.POINTER(C.c_int32)
_f32p = C.POINTER(C.c_float)
_u64p = C.POINTER(C.c_uint64)
_hp = C.c_void_p


def load(path: str | None = None):
    """Load libgpt2q.so; raises if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ImportError(f"libgpt2q.so not built at {p}; run `python -m smelt_b200.build`")
    lib = C.CDLL(p)
    lib.gpt2q_create.argtypes = [C.POINTER(Config), C.POINTER(TensorDesc), C.c_int, C.c_int, C.POINTER(_hp)]
    lib.gpt2q_create.restype = C.c_int
    lib.gpt2q_create_tp.argtypes = [C.POINTER(Config), C.POINTER(TensorDesc), C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_void_p, C.POINTER(_hp)]
    lib.gpt2q_create_tp.restype = C.c_int
    lib.gpt2q_destroy.argtypes = [_hp]
    lib.gpt2q_destroy.restype = None
    lib.gpt2q_last_error.argtypes = [_hp]
    lib.gpt2q_last_error.restype = C.c_char_p
    lib.gpt2q_reset_kv.argtypes = [_hp, _i32p, C.c_int]
    lib.gpt2q_reset_kv.restype = C.c_int
    lib.gpt2q_step.argtypes = [_hp, C.c_uint32, C.c_int32, _f32p]
    lib.gpt2q_step.restype = C.c_int
    # plain addresses: the per-token call path passes array addresses as integers (cheaper than
    # building ctypes pointer objects)
    lib.gpt2q_decode.argtypes = [_hp, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    lib.gpt2q_decode.restype = C.c_int
    lib.gpt2q_prefill.argtypes = [_hp, _u32p, _i32p, _i32p, C.c_int, _f32p, _u32p]
    lib.gpt2q_prefill.restype = C.c_int
    lib.gpt2q_decode_steps.argtypes = [_hp, C.c_int, _u32p]
    lib.gpt2q_decode_steps.restype = C.c_int
    lib.gpt2q_generate_greedy.argtypes = [_hp, _u32p, _i32p, C.c_int, C.c_int, _u32p]
    lib.gpt2q_generate_greedy.restype = C.c_int
    lib.gpt2q_dequant.argtypes = [_hp, C.c_char_p, _f32p, C.c_uint64]
    lib.gpt2q_dequant.restype = C.c_int
    lib.gpt2q_launches.argtypes = [_hp]
    lib.gpt2q_launches.restype = C.c_uint64
    lib.gpt2q_set_stream.argtypes = [_hp, C.c_void_p]
    lib.gpt2q_set_stream.restype = C.c_int
    lib.gpt2q_sync.argtypes = [_hp]
    lib.gpt2q_sync.restype = C.c_int
    lib.gpt2q_set_adapter.argtypes = [_hp, _f32p, _f32p, C.c_int]
    lib.gpt2q_set_adapter.restype = C.c_int
    lib.gpt2q_clear_adapter.argtypes = [_hp]
    lib.gpt2q_clear_adapter.restype = C.c_int
    lib.gpt2q_nll.argtypes = [_hp, _u32p, C.c_int, C.c_int, C.POINTER(C.c_double)]
    lib.gpt2q_nll.restype = C.c_int
    lib.gpt2q_profile.argtypes = [_hp, C.c_int]
    lib.gpt2q_profile.restype = C.c_int
    lib.gpt2q_profile_read.argtypes = [_hp, C.c_char_p, C.c_size_t]
    lib.gpt2q_profile_read.restype = C.c_int
    lib.gpt2q_profile_kernels.argtypes = [_hp, C.c_int, C.c_char_p, C.c_size_t]
    lib.gpt2q_profile_kernels.restype = C.c_int
    lib.gpt2q_info.argtypes = [_hp, C.c_char_p, C.c_size_t]
    lib.gpt2q_info.restype = C.c_int
    lib.gpt2q_argmax_noalloc.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.gpt2q_argmax_noalloc.restype = C.c_int
    lib.gpt2q_rng_new.argtypes = [C.c_uint64]
    lib.gpt2q_rng_new.restype = C.c_uint64
    lib.gpt2q_rng_normal_f32.argtypes = [_u64p, _f32p, C.c_size_t, C.c_double]
    lib.gpt2q_rng_normal_f32.restype = None
    lib.gpt2q_rng_below.argtypes = [_u64p, _u32p, C.c_size_t, C.c_uint64]
    lib.gpt2q_rng_below.restype = None
    lib.gpt2q_create_from_smt.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_hp)]
    lib.gpt2q_create_from_smt.restype = C.c_int
    lib.gpt2q_smt_inspect.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
    lib.gpt2q_smt_inspect.restype = C.c_int
    lib.gpt2q_blake3.argtypes = [C.c_void_p, C.c_uint64, C.POINTER(C.c_uint8)]
    lib.gpt2q_blake3.restype = C.c_int
    lib.gpt2q_trunk_input_grad.argtypes = [_hp, _u32p, C.c_int, _f32p, _f32p, _f32p]
    lib.gpt2q_trunk_input_grad.restype = C.c_int
    lib.gpt2q_bwd_lin_input_grad.argtypes = [C.c_int, _f32p, _f32p, C.c_int, C.c_int, _f32p]
    lib.gpt2q_bwd_lin_input_grad.restype = C.c_int
    lib.gpt2q_bwd_ln_backward.argtypes = [C.c_int, _f32p, _f32p, _f32p, _f32p, C.c_float, C.c_int, _f32p, _f32p,
                                          _f32p]
    lib.gpt2q_bwd_ln_backward.restype = C.c_int
    lib.gpt2q_bwd_gelu.argtypes = [C.c_int, _f32p, _f32p, C.c_int, _f32p]
    lib.gpt2q_bwd_gelu.restype = C.c_int
    lib.gpt2q_bwd_attn_train.argtypes = [C.c_int, _f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p,
                                         _f32p, _f32p]
    lib.gpt2q_bwd_attn_train.restype = C.c_int
    for fn in (lib.gpt2q_quantize_q8, lib.gpt2q_quantize_q4):
        fn.argtypes = [_f32p, C.c_size_t, C.POINTER(C.c_uint8)]
        fn.restype = C.c_int
    if path is None:
        _lib = lib
    return lib


def check(lib, h, rc: int):
    if rc != GPT2Q_OK:
        msg = lib.gpt2q_last_error(h)
        raise Gpt2qError(rc, msg.decode() if msg else "")
