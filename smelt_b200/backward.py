"""Backward ops of the trunk through the C-ABI (the reference's BwdOps, gpu_backward.rs:69-93).

`GpuBwdOps(device)` has the four per-op kernels with host arrays in and out, as GpuBackward's
trait methods (gpu_backward.rs:307-377); `Gpu.trunk_input_grad` (smelt_b200/gpu.py) runs the
whole trunk backward of a sequence on the device.
"""
from __future__ import annotations

import numpy as np

from . import _ffi


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class GpuBwdOps:
    def __init__(self, device: int = 0):
        self._lib = _ffi.load()
        self.device = device

    def _check(self, rc: int):
        _ffi.check(self._lib, None, rc)

    def lin_input_grad(self, w, dy, rows: int, cols: int) -> np.ndarray:
        """dx[i] = sum_r w[r*cols + i] * dy[r]."""
        w, dy = _f32(w), _f32(dy)
        dx = np.empty(cols, np.float32)
        self._check(self._lib.gpt2q_bwd_lin_input_grad(self.device, w.ctypes.data_as(_ffi._f32p),
                                                        dy.ctypes.data_as(_ffi._f32p), rows, cols,
                                                        dx.ctypes.data_as(_ffi._f32p)))
        return dx

    def ln_backward(self, dy, x, g, b, eps, dg=None, db=None):
        """(dx, dg, db); dg/db accumulate into the given arrays (zeros when omitted)."""
        dy, x, g, b = _f32(dy), _f32(x), _f32(g), _f32(b)
        n = x.size
        dx = np.empty(n, np.float32)
        dg = np.zeros(n, np.float32) if dg is None else _f32(dg).copy()
        db = np.zeros(n, np.float32) if db is None else _f32(db).copy()
        p = _ffi._f32p
        self._check(self._lib.gpt2q_bwd_ln_backward(self.device, dy.ctypes.data_as(p), x.ctypes.data_as(p),
                                                     g.ctypes.data_as(p), b.ctypes.data_as(p), float(eps), n,
                                                     dx.ctypes.data_as(p), dg.ctypes.data_as(p), db.ctypes.data_as(p)))
        return dx, dg, db

    def gelu_bwd(self, x, dy) -> np.ndarray:
        x, dy = _f32(x), _f32(dy)
        dx = np.empty(x.size, np.float32)
        p = _ffi._f32p
        self._check(self._lib.gpt2q_bwd_gelu(self.device, x.ctypes.data_as(p), dy.ctypes.data_as(p), x.size,
                                              dx.ctypes.data_as(p)))
        return dx

    def attn_bwd_train(self, q, k, v, dy, t: int, hd: int, stride: int, dk=None, dv=None):
        """(dq, dk, dv); dk/dv accumulate into the given arrays (zeros when omitted)."""
        q, k, v, dy = _f32(q), _f32(k), _f32(v), _f32(dy)
        total = t * stride
        dq = np.empty(total, np.float32)
        dk = np.zeros(total, np.float32) if dk is None else _f32(dk).ravel().copy()
        dv = np.zeros(total, np.float32) if dv is None else _f32(dv).ravel().copy()
        p = _ffi._f32p
        self._check(self._lib.gpt2q_bwd_attn_train(self.device, q.ctypes.data_as(p), k.ctypes.data_as(p),
                                                    v.ctypes.data_as(p), dy.ctypes.data_as(p), t, hd, stride,
                                                    dq.ctypes.data_as(p), dk.ctypes.data_as(p),
                                                    dv.ctypes.data_as(p)))
        return dq, dk, dv
