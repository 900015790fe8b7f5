"""Numeric atoms of the SMT weight format, vectorised with numpy.

Byte-for-byte the encoders of LukasParke/smelt:
  core.f16              experiments/model-lab/src/atoms.rs:10-61 (IEEE half, RNE)
  core.i8.b32.f16scale  atoms.rs:65-78: per 32 values s = amax/127 (fp32, 1.0 when
                        amax == 0); q = clamp(round_half_away(v/s), +-127) with the
                        UNROUNDED s; f16(s) is stored: [f16 LE][32 x int8] = 34 B
  core.i4.b32.f16scale  experiments/perf-lab/src/bin/atoms.rs:89-99 math: d = f16(amax/7)
                        (the ROUNDED d quantises), q = clamp(round_half_away(v/d), +-7).
                        The reference never packs int4; this atom stores
                        [f16 d LE][16 B] with byte j = q[j] & 0xF | (q[j+16] & 0xF) << 4.
"""
from __future__ import annotations

import numpy as np

ATOM_F16 = "core.f16"
ATOM_Q8 = "core.i8.b32.f16scale"
ATOM_Q4 = "core.i4.b32.f16scale"
ATOM_F32 = "core.f32"

Q8_BLOCK = 34
Q4_BLOCK = 18


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """IEEE half bits with round-to-nearest-even (atoms.rs:10-37).

    numpy's float16 cast is the same function for every non-NaN input; NaN maps
    to sign | 0x7d00 as in the reference.
    """
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):
        h = x.astype(np.float16).view(np.uint16).copy()
    nan = np.isnan(x)
    if nan.any():
        sign = (x.view(np.uint32)[nan] >> 16).astype(np.uint16) & 0x8000
        h[nan] = sign | 0x7D00
    return h


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    """Exact half decode (atoms.rs:39-61)."""
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def _round_half_away(r: np.ndarray) -> np.ndarray:
    # Rust f32::round: ties away from zero. r is fp32 with |r| small, exact in f64.
    r64 = r.astype(np.float64)
    return np.where(r64 >= 0, np.floor(r64 + 0.5), -np.floor(-r64 + 0.5))


def _as_i8(v: np.ndarray, lim: int) -> np.ndarray:
    # clamp(round(v/s), +-lim) then Rust `as i8`: NaN (0/0 when a scale underflows) -> 0.
    return np.nan_to_num(np.clip(v, -lim, lim), nan=0.0).astype(np.int8)


def _amax32(x: np.ndarray) -> np.ndarray:
    if np.isnan(x).any():
        raise ValueError("NaN weights cannot be quantised")
    return np.abs(x).max(axis=1)


def q8_encode(x: np.ndarray) -> np.ndarray:
    """Q8 blocks of 32 (atoms.rs:65-78); returns uint8 bytes (n/32 * 34)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if x.size % 32:
        raise ValueError("q8 payload must be a multiple of 32 values")
    b = x.reshape(-1, 32)
    amax = _amax32(b)
    s = np.where(amax == 0, np.float32(1.0), amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = _as_i8(_round_half_away(b / s[:, None]), 127)
    out = np.empty((b.shape[0], Q8_BLOCK), dtype=np.uint8)
    out[:, 0:2] = f32_to_f16_bits(s).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def q4_encode(x: np.ndarray) -> np.ndarray:
    """int4 blocks of 32 (perf-lab atoms.rs:89-99 math); returns uint8 bytes (n/32 * 18)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if x.size % 32:
        raise ValueError("q4 payload must be a multiple of 32 values")
    b = x.reshape(-1, 32)
    amax = _amax32(b)
    dh = f32_to_f16_bits(np.where(amax == 0, np.float32(1.0), amax / np.float32(7.0)).astype(np.float32))
    d = f16_bits_to_f32(dh)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = _as_i8(_round_half_away(b / d[:, None]), 7)
    nib = q.view(np.uint8) & 0x0F
    out = np.empty((b.shape[0], Q4_BLOCK), dtype=np.uint8)
    out[:, 0:2] = dh.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = nib[:, :16] | (nib[:, 16:] << 4)
    return out.reshape(-1)


def _native(fn_name: str, x: np.ndarray, block: int):
    """Run the library's multithreaded quantiser (same bytes as the numpy version)."""
    import ctypes as C

    from . import _ffi

    lib = _ffi.load()
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if x.size % 32:
        raise ValueError("payload must be a multiple of 32 values")
    out = np.empty(x.size // 32 * block, dtype=np.uint8)
    rc = getattr(lib, fn_name)(x.ctypes.data_as(C.POINTER(C.c_float)), x.size, out.ctypes.data_as(C.POINTER(C.c_uint8)))
    if rc != 0:
        raise ValueError(f"{fn_name} failed ({rc})")
    return out


def q8_encode_fast(x: np.ndarray) -> np.ndarray:
    return _native("gpt2q_quantize_q8", x, Q8_BLOCK)


def q4_encode_fast(x: np.ndarray) -> np.ndarray:
    return _native("gpt2q_quantize_q4", x, Q4_BLOCK)


def f16_encode(x: np.ndarray) -> np.ndarray:
    return f32_to_f16_bits(np.ascontiguousarray(x, dtype=np.float32).reshape(-1)).view(np.uint8)


def dequant(atom: str, payload: np.ndarray, numel: int) -> np.ndarray:
    """Host dequantisation, identical to Engine::vec_f32 (gpt2.rs:121-142)."""
    p = np.ascontiguousarray(payload).view(np.uint8)
    if atom == ATOM_F16:
        return f16_bits_to_f32(p.view(np.uint16))[:numel]
    if atom == ATOM_F32:
        return p.view(np.float32)[:numel].copy()
    if atom == ATOM_Q8:
        b = p.reshape(-1, Q8_BLOCK)
        s = f16_bits_to_f32(b[:, :2].copy().view(np.uint16).reshape(-1))
        return (b[:, 2:].view(np.int8).astype(np.float32) * s[:, None]).reshape(-1)[:numel]
    if atom == ATOM_Q4:
        b = p.reshape(-1, Q4_BLOCK)
        s = f16_bits_to_f32(b[:, :2].copy().view(np.uint16).reshape(-1))
        packed = b[:, 2:]
        lo = (packed & 0x0F).astype(np.int16)
        hi = (packed >> 4).astype(np.int16)
        q = np.concatenate([lo, hi], axis=1)
        q = ((q ^ 8) - 8).astype(np.float32)
        return (q * s[:, None]).reshape(-1)[:numel]
    raise ValueError(f"unknown atom {atom}")


def payload_bytes(atom: str, numel: int) -> int:
    return {ATOM_Q8: numel // 32 * Q8_BLOCK, ATOM_Q4: numel // 32 * Q4_BLOCK,
            ATOM_F16: numel * 2, ATOM_F32: numel * 4}[atom]
