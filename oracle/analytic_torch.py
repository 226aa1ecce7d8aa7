"""Test infrastructure: the analytic route as torch fp32 CPU operations, for the timed CPU baseline.

Same steps as `oracle.analytic` (the fp64 numpy form that parity is checked against) in the
precision and operations the reference itself uses on the CPU — fp32, the [H, n, n] score,
softmax and Jacobian matrices materialised, a full SVD for the rank truncation — so that the
baseline runs at the reference's own CPU speed:

* ``rmsnorm_first_order``   src/deltakv/patches/analytic.py:242-262
* ``attention_first_order`` analytic.py:36-98 (GQA by repeating the KV heads, 141-150)
* ``mlp_first_order``       analytic.py:110-138
* ``rank_truncate``         analytic.py:14-22 (returns codes @ basis.T)
* ``analytic_patches``      the engine's loop, src/deltakv/engine.py:377-432

Checked against `oracle.analytic` by `tests/test_oracle_analytic_torch.py`.
"""
from __future__ import annotations

import torch


def rmsnorm_first_order(x, dx, w, eps):
    rms = torch.sqrt((x * x).mean(-1, keepdim=True) + eps)
    y = x / rms * w
    d_rms = (x * dx).mean(-1, keepdim=True) / rms
    dy = (dx * rms - x * d_rms) / (rms * rms) * w
    return y, dy


def rope_tables(hd: int, n: int, base: float):
    inv = 1.0 / (base ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
    f = torch.outer(torch.arange(n, dtype=torch.float32), inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos()[:, None, :], emb.sin()[:, None, :]


def _rope(x, cos, sin):
    h = x.shape[-1] // 2
    return x * cos[: x.shape[0]] + torch.cat([-x[..., h:], x[..., :h]], dim=-1) * sin[: x.shape[0]]


def _apply(fac, x):
    a, b, s = fac
    return ((x @ a.T) * s) @ b.T


def attention_first_order(x, dx, qw, kw, vw, ow, layer, n_heads, n_kv, hd, cos, sin, mask):
    n = x.shape[0]
    q, k, v = ((x @ w.T).view(n, -1, hd) for w in (qw, kw, vw))
    dq, dk, dv = ((dx @ w.T).view(n, -1, hd) for w in (qw, kw, vw))
    if layer:
        for name, t in (("q", dq), ("k", dk), ("v", dv)):
            if name in layer:
                t += _apply(layer[name], x).view(t.shape)
    q, k, dq, dk = (_rope(t, cos, sin) for t in (q, k, dq, dk))
    rep = n_heads // n_kv
    kf, dkf, vf, dvf = (t.repeat_interleave(rep, dim=1).transpose(0, 1) for t in (k, dk, v, dv))
    qh, dqh = q.transpose(0, 1), dq.transpose(0, 1)  # [H, n, hd]
    scale = hd ** -0.5
    a = torch.softmax((qh @ kf.transpose(1, 2)) * scale + mask, dim=-1)
    ds = (dqh @ kf.transpose(1, 2) + qh @ dkf.transpose(1, 2)) * scale
    da = a * (ds - (a * ds).sum(-1, keepdim=True))
    ctx = (a @ vf).transpose(0, 1).reshape(n, -1)
    dctx = (da @ vf + a @ dvf).transpose(0, 1).reshape(n, -1)
    dh = dctx @ ow.T
    if layer and "o" in layer:
        dh = dh + _apply(layer["o"], ctx)
    return dh, dk, dv


def mlp_first_order(x, dx, gw, uw, dw, layer):
    g, u = x @ gw.T, x @ uw.T
    dg, du = dx @ gw.T, dx @ uw.T
    if layer:
        if "gate" in layer:
            dg = dg + _apply(layer["gate"], x)
        if "up" in layer:
            du = du + _apply(layer["up"], x)
    sg = torch.sigmoid(g)
    silu = g * sg
    h = silu * u
    dh = (sg + g * sg * (1.0 - sg)) * dg * u + silu * du
    y = dh @ dw.T
    if layer and "down" in layer:
        y = y + _apply(layer["down"], h)
    return y


def rank_truncate(delta, rank):
    u, s, vh = torch.linalg.svd(delta, full_matrices=False)
    r = max(1, min(rank, s.numel()))
    return (u[:, :r] * s[:r]) @ vh[:r]


def analytic_patches(h, h_mid, weights, layers, cfg):
    """As `oracle.analytic.analytic_patches`, on fp32 tensors; returns ``[(dk, dv)]`` per layer."""
    n = h.shape[1]
    cos, sin = rope_tables(cfg["hd"], n, cfg["rope_base"])
    mask = torch.triu(torch.full((1, n, n), float("-inf")), diagonal=1)
    dx = torch.zeros(n, cfg["d_model"])
    stride = max(1, int(cfg["hidden_stride"]))
    prop_r = max(1, min(int(cfg["propagator_rank"]), cfg["d_model"], n))
    out = []
    for l, w in enumerate(weights):
        if l > 0 and l % stride == 0:
            dx = torch.zeros_like(dx)
        layer = layers.get(l)
        xn, dxn = rmsnorm_first_order(h[l], dx, w["attn_norm"], cfg["eps"])
        dh, dk, dv = attention_first_order(xn, dxn, w["q"], w["k"], w["v"], w["o"], layer, cfg["n_heads"],
                                           cfg["n_kv"], cfg["hd"], cos, sin, mask)
        out.append((dk, dv))
        dx = dx + dh
        xm, dxm = rmsnorm_first_order(h_mid[l], dx, w["mlp_norm"], cfg["eps"])
        dx = dx + mlp_first_order(xm, dxm, w["gate"], w["up"], w["down"], layer)
        dx = rank_truncate(dx, prop_r)
    return out
