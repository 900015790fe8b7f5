"""CPU restatement of the reference's trunk backward (the plasticity path), in float64.

TEST INFRASTRUCTURE ONLY: the checker the library's backward kernels (smelt_b200/csrc/
backward.cu, gpt2q_trunk_input_grad in runtime.cu) are compared against. Only tests/ import it.

* ``Rng``: xorshift64* of experiments/model-lab/src/gpu_backward.rs:835-858 (f32 uniform in
  [-1, 1), below).
* ``selfcheck``: the finite-difference self-checks of each backward kernel
  (gpu_backward.rs:915-1090, same seeds, sizes and tolerances, ``rel_max`` of :860-872), run
  through any implementation of the four ops.
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
def selfcheck(ops, which: str):
    """gpu_backward.rs:915-1090 through `ops` (an object with lin_input_grad(w, dy, rows, cols),
    ln_backward(dy, x, g, b, eps) -> (dx, dg, db), gelu_bwd(x, dy), attn_bwd_train(q, k, v, dy,
    t, hd, stride) -> (dq, dk, dv), all float32 in and out). Returns (max_rel, tol)."""
    if which == "k_lin_input_grad":
        r = Rng(101)
        rows, cols = 16, 24
        w = np.array([r.f32() for _ in range(rows * cols)], np.float32)
        c = np.array([r.f32() for _ in range(rows)], np.float32)
        dx = ops.lin_input_grad(w, c, rows, cols)
        wf, cf = w.astype(np.float64).reshape(rows, cols), c.astype(np.float64)
        h = 1e-5
        fd = np.zeros(cols)
        y = np.zeros(cols)
        for i in range(cols):
            y[i] += h
            lp = float(cf @ (wf @ y))
            y[i] -= 2 * h
            lm = float(cf @ (wf @ y))
            y[i] += h
            fd[i] = (lp - lm) / (2 * h)
        return rel_max(dx, fd.astype(np.float32)), 1e-4
    if which == "k_ln_backward":
        r = Rng(202)
        n, eps = 64, np.float32(1e-5)
        x0 = np.array([r.f32() for _ in range(n)], np.float32)
        g0 = np.array([r.f32() for _ in range(n)], np.float32)
        b0 = np.array([r.f32() for _ in range(n)], np.float32)
        dy0 = np.array([r.f32() for _ in range(n)], np.float32).astype(np.float64)
        dx, dg, db = ops.ln_backward(dy0.astype(np.float32), x0, g0, b0, eps)

        def df(xx, gg, bb):
            mean = xx.sum() / n
            var = ((xx - mean) ** 2).sum() / n
            return float((((xx - mean) / np.sqrt(var + float(eps)) * gg + bb) * dy0).sum())

        xf, gf, bf = (a.astype(np.float64) for a in (x0, g0, b0))
        h = 1e-6

        def fd_of(which_arr):
            out = np.zeros(n, np.float32)
            arrs = [xf.copy(), gf.copy(), bf.copy()]
            a = arrs[which_arr]
            for i in range(n):
                keep = a[i]
                a[i] = keep + h
                lp = df(*arrs)
                a[i] = keep - h
                lm = df(*arrs)
                a[i] = keep
                out[i] = np.float32((lp - lm) / (2 * h))
            return out

        mr = max(rel_max(dx, fd_of(0)), rel_max(dg, fd_of(1)), rel_max(db, fd_of(2)))
        return mr, 1e-3
    if which == "k_gelu_bwd":
        r = Rng(303)
        n = 32
        xp = np.array([np.float32(r.f32() * np.float32(3.0)) for _ in range(n)], np.float32)
        dy0 = np.array([r.f32() for _ in range(n)], np.float32).astype(np.float64)
        dx = ops.gelu_bwd(xp, dy0.astype(np.float32))
        xx = xp.astype(np.float64)
        h = 1e-6
        fd = np.zeros(n)
        for i in range(n):
            xx[i] += h
            lp = float((gelu(xx) * dy0).sum())
            xx[i] -= 2 * h
            lm = float((gelu(xx) * dy0).sum())
            xx[i] += h
            fd[i] = (lp - lm) / (2 * h)
        return rel_max(dx, fd.astype(np.float32)), 1e-3
    if which == "k_attn_bwd_train":
        r = Rng(404)
        t_len, hd, stride = 5, 8, 8
        total = t_len * stride
        q = np.array([r.f32() for _ in range(total)], np.float32)
        k = np.array([r.f32() for _ in range(total)], np.float32)
        v = np.array([r.f32() for _ in range(total)], np.float32)
        dy0 = np.array([r.f32() for _ in range(total)], np.float32)
        dq, dk, dv = ops.attn_bwd_train(q, k, v, dy0, t_len, hd, stride)

        def f(qq, kk, vv):
            o = attn_causal(qq.astype(np.float64).reshape(t_len, stride), kk.astype(np.float64).reshape(t_len, stride),
                            vv.astype(np.float64).reshape(t_len, stride), stride // hd)
            return float((o.ravel() * dy0.astype(np.float64)).sum())

        h = np.float32(1e-4)

        def fd_of(arr, pos):
            out = np.zeros(total, np.float32)
            a = arr.copy()
            for i in range(total):
                keep = a[i]
                a[i] = np.float32(keep + h)
                args = [q, k, v]
                args[pos] = a
                lp = f(*args)
                a[i] = np.float32(np.float32(keep + h) - np.float32(2.0) * h)
                args[pos] = a
                lm = f(*args)
                a[i] = keep
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
