"""Oracle of the analytic route (numpy, fp64; TEST INFRASTRUCTURE ONLY — never on the product
path).

Restates src/deltakv/patches/analytic.py and the engine's per-layer loop
(src/deltakv/engine.py:377-432) on materialised matrices:

* ``rmsnorm_first_order``  analytic.py:245-262
* ``rope``                 rope.py:9-63 (rotate-half, positions 0..n-1)
* ``attention_first_order`` analytic.py:38-95 (GQA by repeating kv heads, 141-153)
* ``mlp_first_order``      analytic.py:108-138
* ``rank_truncate``        analytic.py:14-22 (returns codes @ basis.T)
* ``analytic_patches``     engine.py:377-432
"""

from __future__ import annotations

import numpy as np


def rmsnorm_first_order(x, dx, w, eps):
    x, dx, w = (np.asarray(a, np.float64) for a in (x, dx, w))
    rms = np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    y = x / rms * w
    d_rms = 0.5 * (2.0 * (x * dx).mean(-1, keepdims=True)) / rms
    dy = (dx * rms - x * d_rms) / (rms * rms) * w
    return y, dy


def rope_tables(hd: int, n: int, base: float):
    inv = 1.0 / (base ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    f = np.outer(np.arange(n, dtype=np.float64), inv)
    emb = np.concatenate([f, f], axis=-1)
    return np.cos(emb), np.sin(emb)


def rope(x, cos, sin):
    """``x [n, heads, hd]`` at positions 0..n-1."""
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return x * cos[: x.shape[0], None, :] + rot * sin[: x.shape[0], None, :]


def _apply(fac, x):
    a, b, s = fac
    return (s * (x @ a.T)) @ b.T


def attention_first_order(x, dx, qw, kw, vw, ow, layer, n_heads, n_kv, hd, cos, sin):
    n = x.shape[0]
    f = lambda m, w: (m @ np.asarray(w, np.float64).T)
    q, k, v = (f(x, w).reshape(n, -1, hd) for w in (qw, kw, vw))
    dq, dk, dv = (f(dx, w).reshape(n, -1, hd) for w in (qw, kw, vw))
    if layer:
        for name, t in (("q", dq), ("k", dk), ("v", dv)):
            if name in layer:
                t += _apply(layer[name], x).reshape(t.shape)
    q, k, dq, dk = (rope(t, cos, sin) for t in (q, k, dq, dk))
    rep = n_heads // n_kv
    kf, dkf, vf, dvf = (np.repeat(t, rep, axis=1) for t in (k, dk, v, dv))
    scale = hd ** -0.5
    s = np.einsum("qhd,khd->hqk", q, kf) * scale
    mask = np.triu(np.full((n, n), -np.inf), 1)
    s = s + mask
    s = s - s.max(-1, keepdims=True)
    a = np.exp(s)
    a /= a.sum(-1, keepdims=True)
    ds = (np.einsum("qhd,khd->hqk", dq, kf) + np.einsum("qhd,khd->hqk", q, dkf)) * scale
    da = a * (ds - (a * ds).sum(-1, keepdims=True))
    ctx = np.einsum("hqk,khd->qhd", a, vf)
    dctx = np.einsum("hqk,khd->qhd", da, vf) + np.einsum("hqk,khd->qhd", a, dvf)
    dh = dctx.reshape(n, -1) @ np.asarray(ow, np.float64).T
    if layer and "o" in layer:
        dh = dh + _apply(layer["o"], ctx.reshape(n, -1))
    return dh, dk, dv


def _silu(x):
    return x / (1.0 + np.exp(-x))


def mlp_first_order(x, dx, gw, uw, dw, layer):
    g, u = x @ np.asarray(gw, np.float64).T, x @ np.asarray(uw, np.float64).T
    dg, du = dx @ np.asarray(gw, np.float64).T, dx @ np.asarray(uw, np.float64).T
    if layer:
        if "gate" in layer:
            dg = dg + _apply(layer["gate"], x)
        if "up" in layer:
            du = du + _apply(layer["up"], x)
    sg = 1.0 / (1.0 + np.exp(-g))
    h = _silu(g) * u
    dh = (sg + g * sg * (1.0 - sg)) * dg * u + _silu(g) * du
    y = dh @ np.asarray(dw, np.float64).T
    if layer and "down" in layer:
        y = y + _apply(layer["down"], h)
    return y


def rank_truncate(delta, rank):
    u, s, vh = np.linalg.svd(delta, full_matrices=False)
    r = max(1, min(rank, s.size))
    return (u[:, :r] * s[:r]) @ vh[:r]


def analytic_patches(h, h_mid, weights, layers, cfg):
    """``weights[l]``: dict of q, k, v, o, gate, up, down, attn_norm, mlp_norm arrays;
    ``layers[l]``: dict projection -> (A, B, scale) or absent; ``cfg``: n_heads, n_kv, hd,
    d_model, eps, rope_base, hidden_stride, propagator_rank.  Returns ``[(dk, dv)]`` per layer."""
    n = h.shape[1]
    cos, sin = rope_tables(cfg["hd"], n, cfg["rope_base"])
    dx = np.zeros((n, cfg["d_model"]))
    stride = max(1, int(cfg["hidden_stride"]))
    prop_r = max(1, min(int(cfg["propagator_rank"]), cfg["d_model"], n))
    out = []
    for l, w in enumerate(weights):
        if l > 0 and l % stride == 0:
            dx = np.zeros_like(dx)
        layer = layers.get(l)
        xn, dxn = rmsnorm_first_order(h[l], dx, w["attn_norm"], cfg["eps"])
        dh, dk, dv = attention_first_order(xn, dxn, w["q"], w["k"], w["v"], w["o"], layer, cfg["n_heads"],
                                           cfg["n_kv"], cfg["hd"], cos, sin)
        out.append((dk, dv))
        dx = dx + dh
        xm, dxm = rmsnorm_first_order(h_mid[l], dx, w["mlp_norm"], cfg["eps"])
        dx = dx + mlp_first_order(xm, dxm, w["gate"], w["up"], w["down"], layer)
        dx = rank_truncate(dx, prop_r)
    return out
