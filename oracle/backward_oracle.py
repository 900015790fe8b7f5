"""CPU restatement of the reference's trunk backward (the plasticity path), in float64.

TEST INFRASTRUCTURE ONLY: the checker the library's backward kernels (smelt_b200/csrc/
backward.cu, gpt2q_trunk_input_grad in runtime.cu) are compared against. Only tests/ import it.

* ``Rng``: xorshift64* of experiments/model-lab/src/gpu_backward.rs:835-858 (f32 uniform in
  [-1, 1), below).
* ``selfcheck``: the finite-difference self-checks of each backward kernel
  (gpu_backward.rs:915-1090, same seeds, sizes and tolerances, ``rel_max`` of :860-872), run
  through any implementation of the four ops. The finite-difference side keeps the reference's
  evaluation order (sequential f64 sums), so that ``MirrorOps32`` (the reference's CPU mirror,
  gpu_backward.rs:450-590, in f32 with Rust's operation order) prints the reference's own
  logged KCHECK lines digit for digit (docs/experiments/results/bwparity.log:6-9): the pin of
  the Rng, the harness and rel_max.
* ``forward_stash``: the stash of bin/bwparity.rs forward_stash (:448-580): per layer the residual
  entering the layer, the residual after attention, q|k|v with bias, the pre-GELU c_fc output;
  the input and output of ln_f; the logits.
* ``trunk_input_grad``: gpu_backward.rs:651-790 with the MirrorOps math (:450-590), every
  position at once.
* ``fd_embedding_check``: bwparity.rs:690-735: central differences of the linear readout loss
  sum(dlogits * logits) with respect to sampled wte coordinates, against the analytic input
  path (dx at the positions holding that token) plus the tied-head path.
Everything is float64 over the exactly dequantised weights (Engine::vec_f32).
"""
from __future__ import annotations

import math
import sys

import numpy as np

M64 = (1 << 64) - 1


class Rng:
    """gpu_backward.rs:835-858."""

    def __init__(self, seed: int):
        self.s = (seed ^ 0x9E3779B97F4A7C15) & M64

    def next_u64(self) -> int:
        x = self.s
        x ^= x >> 12
        x ^= (x << 25) & M64
        x ^= x >> 27
        self.s = x
        return (x * 0x2545F4914F6CDD1D) & M64

    def f32(self) -> np.float32:
        return np.float32(np.float32((self.next_u64() >> 40) / float(1 << 24)) * np.float32(2.0) - np.float32(1.0))

    def below(self, n: int) -> int:
        return self.next_u64() % n


def rel_max(a, fd) -> float:
    """gpu_backward.rs:860-872: max |a-f| / max(|a|, |f|, 1e-3 * max|f|)."""
    a = np.asarray(a, np.float64).ravel()
    f = np.asarray(fd, np.float64).ravel()
    fscale = max(np.max(np.abs(f)) if f.size else 0.0, 1e-30) * 1e-3
    den = np.maximum(np.maximum(np.abs(a), np.abs(f)), fscale)
    return float(np.max(np.abs(a - f) / den)) if a.size else 0.0


# ---------------------------------------------------------------- f64 forward pieces
def gelu(v):
    return 0.5 * v * (1.0 + np.tanh(0.7978845608028654 * (v + 0.044715 * v * v * v)))


def layernorm(x, g, b, eps):
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return (x - mean) / np.sqrt(var + eps) * g + b


def attn_causal(q, k, v, n_head):
    """Training-form causal attention over [T, E] q/k/v (gpu_backward.rs f64ref::attn_add)."""
    T, E = q.shape
    hd = E // n_head
    out = np.zeros_like(q)
    mask = np.tril(np.ones((T, T), bool))
    for h in range(n_head):
        sl = slice(h * hd, (h + 1) * hd)
        s = (q[:, sl] @ k[:, sl].T) / np.sqrt(hd)
        s = np.where(mask, s, -np.inf)
        s = np.exp(s - s.max(axis=1, keepdims=True))
        p = s / s.sum(axis=1, keepdims=True)
        out[:, sl] = p @ v[:, sl]
    return out


def weights64(pack) -> dict:
    """Every tensor of the pack dequantised (exact) and widened to float64."""
    return {n: pack.dequant(n).astype(np.float64) for n in pack.tensors}


def forward_stash(W: dict, meta, ids, wte=None):
    """bwparity.rs forward_stash (:448-580) in f64; returns (logits [T][V], acts)."""
    wte = W["wte.weight"] if wte is None else wte
    T, E = len(ids), meta.n_embd
    x = wte[np.asarray(ids)] + W["wpe.weight"][:T]
    acts = {"x_in": [], "x_mid": [], "qkv": [], "fc_pre": []}
    for l in range(meta.n_layer):
        p = f"h.{l}."
        acts["x_in"].append(x.copy())
        h1 = layernorm(x, W[p + "ln_1.weight"], W[p + "ln_1.bias"], meta.ln_eps)
        qkv = h1 @ W[p + "attn.c_attn.weight"].T + W[p + "attn.c_attn.bias"]
        acts["qkv"].append(qkv)
        a = attn_causal(qkv[:, :E], qkv[:, E:2 * E], qkv[:, 2 * E:], meta.n_head)
        x = x + a @ W[p + "attn.c_proj.weight"].T + W[p + "attn.c_proj.bias"]
        acts["x_mid"].append(x.copy())
        h2 = layernorm(x, W[p + "ln_2.weight"], W[p + "ln_2.bias"], meta.ln_eps)
        fc = h2 @ W[p + "mlp.c_fc.weight"].T + W[p + "mlp.c_fc.bias"]
        acts["fc_pre"].append(fc)
        x = x + gelu(fc) @ W[p + "mlp.c_proj.weight"].T + W[p + "mlp.c_proj.bias"]
    acts["lnf_x"] = x.copy()
    lnf = layernorm(x, W["ln_f.weight"], W["ln_f.bias"], meta.ln_eps)
    acts["lnf_out"] = lnf
    return lnf @ wte.T, acts


# ---------------------------------------------------------------- MirrorOps (f64, batched)
def lin_input_grad(w, dy):
    """dx[i] = sum_r w[r][i] dy[r] (MirrorOps::lin_input_grad, :452-463), rows of dy batched."""
    return dy @ w


def ln_backward(dy, x, g, eps):
    """MirrorOps::ln_backward (:465-492) per row; returns (dx, dg, db) with dg/db summed."""
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(var + eps)
    xh = (x - mean) * rstd
    dh = dy * g
    mdxh = dh.mean(axis=-1, keepdims=True)
    mdxh_xh = (dh * xh).mean(axis=-1, keepdims=True)
    dx = rstd * (dh - mdxh - xh * mdxh_xh)
    return dx, (dy * xh).sum(axis=0), dy.sum(axis=0)


def gelu_bwd(x, dy):
    """MirrorOps::gelu_bwd (:494-506)."""
    u = 0.7978845608028654 * (x + 0.044715 * x * x * x)
    th = np.tanh(u)
    sech2 = 1.0 - th * th
    return dy * (0.5 * (1.0 + th) + 0.5 * x * sech2 * 0.7978845608028654 * (1.0 + 3.0 * 0.044715 * x * x))


def attn_bwd_train(q, k, v, dy, hd):
    """MirrorOps::attn_bwd_train (:508-590) over [T, stride] arrays; returns (dq, dk, dv)."""
    T, stride = q.shape
    dq, dk, dv = np.zeros_like(q), np.zeros_like(q), np.zeros_like(q)
    scale = 1.0 / np.sqrt(hd)
    mask = np.tril(np.ones((T, T), bool))
    for h in range(stride // hd):
        sl = slice(h * hd, (h + 1) * hd)
        s = np.where(mask, (q[:, sl] @ k[:, sl].T) * scale, -np.inf)
        s = np.exp(s - s.max(axis=1, keepdims=True))
        p = s / s.sum(axis=1, keepdims=True)
        dp = np.where(mask, dy[:, sl] @ v[:, sl].T, 0.0)
        rs = (dp * p).sum(axis=1, keepdims=True)
        ds = (dp - rs) * p * scale
        dq[:, sl] = ds @ k[:, sl]
        dk[:, sl] = ds.T @ q[:, sl]
        dv[:, sl] = p.T @ dy[:, sl]
    return dq, dk, dv


def trunk_input_grad(W: dict, meta, acts, dlogits):
    """gpu_backward.rs:651-790: dlogits [T][V] -> dx [T][E] at the embedding output."""
    E = meta.n_embd
    hd = E // meta.n_head
    dh = lin_input_grad(W["wte.weight"], dlogits)
    g, _, _ = ln_backward(dh, acts["lnf_x"], W["ln_f.weight"], meta.ln_eps)
    for l in reversed(range(meta.n_layer)):
        p = f"h.{l}."
        d_fc = gelu_bwd(acts["fc_pre"][l], lin_input_grad(W[p + "mlp.c_proj.weight"], g))
        dh2 = lin_input_grad(W[p + "mlp.c_fc.weight"], d_fc)
        dxl2, _, _ = ln_backward(dh2, acts["x_mid"][l], W[p + "ln_2.weight"], meta.ln_eps)
        combined = g + dxl2
        dattn = lin_input_grad(W[p + "attn.c_proj.weight"], combined)
        qkv = acts["qkv"][l]
        dq, dk, dv = attn_bwd_train(qkv[:, :E], qkv[:, E:2 * E], qkv[:, 2 * E:], dattn, hd)
        dh1 = lin_input_grad(W[p + "attn.c_attn.weight"], np.concatenate([dq, dk, dv], axis=1))
        dxl1, _, _ = ln_backward(dh1, acts["x_in"][l], W[p + "ln_1.weight"], meta.ln_eps)
        g = g + dxl1 + dxl2
    return g


def sparse_dlogits(T: int, vocab: int, seed: int = 20260824) -> np.ndarray:
    """bwparity.rs:599-607: 8 random (index, uniform value) entries per position."""
    rng = Rng(seed)
    out = np.zeros((T, vocab), np.float32)
    for p in range(T):
        for _ in range(8):
            idx = rng.below(vocab)
            out[p, idx] = rng.f32()
    return out


def fd_embedding_check(W: dict, meta, ids, dlogits, dx, lnf_out, n_coords: int = 32, rel_delta: float = 1e-2):
    """bwparity.rs:690-735: (analytic, fd) per sampled wte coordinate; analytic = the input
    path sum_{p: ids[p]==tok} dx[p][idx] plus the tied-head path sum_p dlogits[p][tok] lnf_out[p][idx]."""
    T = len(ids)
    wte = W["wte.weight"].copy()
    dl64 = np.asarray(dlogits, np.float64)
    rows = []
    for c in range(n_coords):
        ti = c % T
        tok = int(ids[ti])
        idx = (c * 97 + 13) % meta.n_embd
        v0 = wte[tok, idx]
        h = rel_delta * max(abs(v0), 0.05)
        wte[tok, idx] = v0 + h
        lp = float((dl64 * forward_stash(W, meta, ids, wte)[0]).sum())
        wte[tok, idx] = v0 - h
        lm = float((dl64 * forward_stash(W, meta, ids, wte)[0]).sum())
        wte[tok, idx] = v0
        fd = (lp - lm) / (2 * h)
        inp = sum(float(dx[p][idx]) for p in range(T) if int(ids[p]) == tok)
        head = sum(float(dlogits[p][tok]) * float(lnf_out[p][idx]) for p in range(T))
        rows.append((inp + head, fd))
    return np.array(rows)


# ---------------------------------------------------------------- kernel self-checks
# f64 reference forwards of the self-checks, evaluated in the reference's order (sequential
# iterator sums, libm transcendentals), so the finite differences carry the same rounding
def _seq_sum(vals) -> float:
    s = 0.0
    for v in vals:
        s += v
    return s


def _f64_gelu(v: float) -> float:
    return 0.5 * v * (1.0 + math.tanh(0.7978845608028654 * (v + 0.044715 * v * v * v)))


def _f64_attn_add(q, k, v, t_len, hd, stride, out):
    """gpu_backward.rs f64ref::attn_add: causal training-form attention, adds into out."""
    scale = 1.0 / math.sqrt(hd)
    for head in range(stride // hd):
        base = head * hd
        for i in range(t_len):
            scores = []
            for j in range(i + 1):
                d = 0.0
                for tt in range(hd):
                    d += float(q[i * stride + base + tt]) * float(k[j * stride + base + tt])
                scores.append(d * scale)
            mx = -sys.float_info.max
            for sc in scores:
                mx = max(mx, sc)
            ssum = 0.0
            for j in range(len(scores)):
                scores[j] = math.exp(scores[j] - mx)
                ssum += scores[j]
            for j in range(len(scores)):
                scores[j] /= ssum
            for j in range(i + 1):
                for tt in range(hd):
                    out[i * stride + base + tt] += scores[j] * float(v[j * stride + base + tt])


def selfcheck(ops, which: str):
    """gpu_backward.rs:915-1090 through `ops` (an object with lin_input_grad(w, dy, rows, cols),
    ln_backward(dy, x, g, b, eps) -> (dx, dg, db), gelu_bwd(x, dy), attn_bwd_train(q, k, v, dy,
    t, hd, stride) -> (dq, dk, dv), all float32 in and out). Returns (max_rel, tol). The f64 side
    follows the reference's evaluation order, so MirrorOps32 reproduces the reference's logged
    KCHECK values for its CPU mirror."""
    if which == "k_lin_input_grad":
        r = Rng(101)
        rows, cols = 16, 24
        w = np.array([r.f32() for _ in range(rows * cols)], np.float32)
        c = np.array([r.f32() for _ in range(rows)], np.float32)
        dx = ops.lin_input_grad(w, c, rows, cols)
        wf = [float(v) for v in w]
        cf = [float(v) for v in c]
        h = 1e-5

        def f(y):
            acc = 0.0
            for rr in range(rows):
                d = 0.0
                for j in range(cols):
                    d += wf[rr * cols + j] * y[j]
                acc += cf[rr] * d
            return acc

        y = [0.0] * cols
        fd = np.zeros(cols, np.float32)
        for i in range(cols):
            y[i] += h
            lp = f(y)
            y[i] -= 2.0 * h
            lm = f(y)
            y[i] += h
            fd[i] = np.float32((lp - lm) / (2.0 * h))
        return rel_max(dx, fd), 1e-4
    if which == "k_ln_backward":
        r = Rng(202)
        n, eps = 64, np.float32(1e-5)
        x0 = np.array([r.f32() for _ in range(n)], np.float32)
        g0 = np.array([r.f32() for _ in range(n)], np.float32)
        b0 = np.array([r.f32() for _ in range(n)], np.float32)
        dy0 = [float(r.f32()) for _ in range(n)]
        dx, dg, db = ops.ln_backward(np.array(dy0, np.float32), x0, g0, b0, eps)

        def df(xx, gg, bb):
            mean = _seq_sum(xx) / n
            var = _seq_sum((v - mean) * (v - mean) for v in xx) / n
            den = math.sqrt(var + float(eps))
            return _seq_sum(((xx[i] - mean) / den * gg[i] + bb[i]) * dy0[i] for i in range(n))

        base = [[float(v) for v in a] for a in (x0, g0, b0)]
        h = 1e-6

        def fd_of(which_arr):
            arrs = [list(a) for a in base]
            a = arrs[which_arr]
            out = np.zeros(n, np.float32)
            for i in range(n):
                keep = a[i]
                a[i] = keep + h
                lp = df(*arrs)
                a[i] = keep - h
                lm = df(*arrs)
                a[i] = keep
                out[i] = np.float32((lp - lm) / (2.0 * h))
            return out

        mr = max(rel_max(dx, fd_of(0)), rel_max(dg, fd_of(1)), rel_max(db, fd_of(2)))
        return mr, 1e-3
    if which == "k_gelu_bwd":
        r = Rng(303)
        n = 32
        xp = np.array([np.float32(r.f32() * np.float32(3.0)) for _ in range(n)], np.float32)
        dy0 = [float(r.f32()) for _ in range(n)]
        dx = ops.gelu_bwd(xp, np.array(dy0, np.float32))
        xx = [float(v) for v in xp]
        h = 1e-6
        fd = np.zeros(n, np.float32)
        for i in range(n):
            xx[i] += h
            lp = _seq_sum(_f64_gelu(v) * d for v, d in zip(xx, dy0))
            xx[i] -= 2.0 * h
            lm = _seq_sum(_f64_gelu(v) * d for v, d in zip(xx, dy0))
            xx[i] += h
            fd[i] = np.float32((lp - lm) / (2.0 * h))
        return rel_max(dx, fd), 1e-3
    if which == "k_attn_bwd_train":
        r = Rng(404)
        t_len, hd, stride = 5, 8, 8
        total = t_len * stride
        q = np.array([r.f32() for _ in range(total)], np.float32)
        k = np.array([r.f32() for _ in range(total)], np.float32)
        v = np.array([r.f32() for _ in range(total)], np.float32)
        dy0 = np.array([r.f32() for _ in range(total)], np.float32)
        dq, dk, dv = ops.attn_bwd_train(q, k, v, dy0, t_len, hd, stride)
        dyl = [float(x) for x in dy0]

        def f(qq, kk, vv):
            out = [0.0] * total
            _f64_attn_add(qq, kk, vv, t_len, hd, stride, out)
            return _seq_sum(a * d for a, d in zip(out, dyl))

        h = np.float32(1e-4)

        def fd_of(arr, pos):
            out = np.zeros(total, np.float32)
            a = arr.copy()
            for i in range(total):
                a[i] = np.float32(a[i] + h)
                args = [q, k, v]
                args[pos] = a
                lp = f(*args)
                a[i] = np.float32(a[i] - np.float32(2.0) * h)
                lm = f(*args)
                a[i] = np.float32(a[i] + h)
                out[i] = np.float32((lp - lm) / (2.0 * float(h)))
            return out

        mr = max(rel_max(dq, fd_of(q, 0)), rel_max(dk, fd_of(k, 1)), rel_max(dv, fd_of(v, 2)))
        return mr, 1e-2
    raise ValueError(which)


KERNELS = ("k_lin_input_grad", "k_ln_backward", "k_gelu_bwd", "k_attn_bwd_train")


class MirrorOps:
    """The oracle's own four ops (float32 in/out), for checking the self-check harness."""

    def lin_input_grad(self, w, dy, rows, cols):
        return lin_input_grad(w.astype(np.float64).reshape(rows, cols), dy.astype(np.float64)).astype(np.float32)

    def ln_backward(self, dy, x, g, b, eps):
        dx, dg, db = ln_backward(dy.astype(np.float64)[None], x.astype(np.float64)[None], g.astype(np.float64),
                                 float(eps))
        return dx[0].astype(np.float32), dg.astype(np.float32), db.astype(np.float32)

    def gelu_bwd(self, x, dy):
        return gelu_bwd(x.astype(np.float64), dy.astype(np.float64)).astype(np.float32)

    def attn_bwd_train(self, q, k, v, dy, t, hd, stride):
        sh = (t, stride)
        out = attn_bwd_train(*(a.astype(np.float64).reshape(sh) for a in (q, k, v, dy)), hd)
        return tuple(o.ravel().astype(np.float32) for o in out)


class MirrorOps32:
    """MirrorOps (gpu_backward.rs:450-590) in float32 with the Rust operation order: sequential
    sums, separate multiply and add (Rust does not fuse), f32 transcendentals. Pure-Python
    loops: only for the self-check sizes."""

    def lin_input_grad(self, w, dy, rows, cols):
        w = np.asarray(w, np.float32).reshape(rows, cols)
        dy = np.asarray(dy, np.float32)
        dx = np.zeros(cols, np.float32)
        for i in range(cols):
            acc = np.float32(0.0)
            for r in range(rows):
                acc = np.float32(acc + np.float32(w[r, i] * dy[r]))
            dx[i] = acc
        return dx

    def ln_backward(self, dy, x, g, b, eps):
        dy, x, g = (np.asarray(a, np.float32) for a in (dy, x, g))
        n = x.size
        nf = np.float32(n)
        s = np.float32(0.0)
        for v in x:
            s = np.float32(s + v)
        mean = np.float32(s / nf)
        sq = np.float32(0.0)
        for v in x:
            d = np.float32(v - mean)
            sq = np.float32(sq + np.float32(d * d))
        var = np.float32(sq / nf)
        rstd = np.float32(np.float32(1.0) / np.sqrt(np.float32(var + np.float32(eps))))
        mdxh = np.float32(0.0)
        mdxh_xh = np.float32(0.0)
        for i in range(n):
            dh = np.float32(dy[i] * g[i])
            mdxh = np.float32(mdxh + dh)
            mdxh_xh = np.float32(mdxh_xh + np.float32(np.float32(dh * np.float32(x[i] - mean)) * rstd))
        mdxh = np.float32(mdxh / nf)
        mdxh_xh = np.float32(mdxh_xh / nf)
        dx = np.zeros(n, np.float32)
        dg = np.zeros(n, np.float32)
        db = np.zeros(n, np.float32)
        for i in range(n):
            xh = np.float32(np.float32(x[i] - mean) * rstd)
            dh = np.float32(dy[i] * g[i])
            dx[i] = np.float32(rstd * np.float32(np.float32(dh - mdxh) - np.float32(xh * mdxh_xh)))
            dg[i] = np.float32(dg[i] + np.float32(dy[i] * xh))
            db[i] = np.float32(db[i] + dy[i])
        return dx, dg, db

    def gelu_bwd(self, x, dy):
        x, dy = np.asarray(x, np.float32), np.asarray(dy, np.float32)
        c, k = np.float32(0.7978845608028654), np.float32(0.044715)
        dx = np.zeros(x.size, np.float32)
        for i in range(x.size):
            v = x[i]
            u = np.float32(c * np.float32(v + np.float32(np.float32(np.float32(k * v) * v) * v)))
            th = np.float32(np.tanh(u))
            sech2 = np.float32(np.float32(1.0) - np.float32(th * th))
            t1 = np.float32(np.float32(0.5) * np.float32(np.float32(1.0) + th))
            t2 = np.float32(np.float32(np.float32(np.float32(np.float32(0.5) * v) * sech2) * c) *
                            np.float32(np.float32(1.0) + np.float32(np.float32(np.float32(np.float32(3.0) * k) * v) * v)))
            dx[i] = np.float32(dy[i] * np.float32(t1 + t2))
        return dx

    def attn_bwd_train(self, q, k, v, dy, t, hd, stride):
        q, k, v, dy = (np.asarray(a, np.float32).reshape(-1) for a in (q, k, v, dy))
        total = t * stride
        dq, dk, dv = np.zeros(total, np.float32), np.zeros(total, np.float32), np.zeros(total, np.float32)
        scale = np.float32(np.float32(1.0) / np.sqrt(np.float32(hd)))
        for head in range(stride // hd):
            base = head * hd
            for i in range(t):
                scores = []
                mx = np.float32(np.finfo(np.float32).min)
                for j in range(i + 1):
                    d = np.float32(0.0)
                    for tt in range(hd):
                        d = np.float32(d + np.float32(q[i * stride + base + tt] * k[j * stride + base + tt]))
                    s = np.float32(d * scale)
                    scores.append(s)
                    mx = max(mx, s)
                ssum = np.float32(0.0)
                for j in range(i + 1):
                    scores[j] = np.float32(np.exp(np.float32(scores[j] - mx)))
                    ssum = np.float32(ssum + scores[j])
                for j in range(i + 1):
                    scores[j] = np.float32(scores[j] / ssum)
                dp = []
                rs = np.float32(0.0)
                for j in range(i + 1):
                    d = np.float32(0.0)
                    for tt in range(hd):
                        d = np.float32(d + np.float32(dy[i * stride + base + tt] * v[j * stride + base + tt]))
                    dp.append(d)
                    rs = np.float32(rs + np.float32(d * scores[j]))
                ds = [np.float32(np.float32(np.float32(dp[j] - rs) * scores[j]) * scale) for j in range(i + 1)]
                for tt in range(hd):
                    acc = np.float32(0.0)
                    for j in range(i + 1):
                        acc = np.float32(acc + np.float32(ds[j] * k[j * stride + base + tt]))
                    dq[i * stride + base + tt] = acc
                for j in range(i + 1):
                    for tt in range(hd):
                        dk[j * stride + base + tt] = np.float32(dk[j * stride + base + tt] +
                                                                np.float32(ds[j] * q[i * stride + base + tt]))
                        dv[j * stride + base + tt] = np.float32(dv[j * stride + base + tt] +
                                                                np.float32(scores[j] * dy[i * stride + base + tt]))
        return dq, dk, dv
