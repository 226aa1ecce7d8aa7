"""Oracle restatement of the toy decoder (numpy fp32; TEST INFRASTRUCTURE ONLY): the full
prefill that produces the stored activations and the cached K/V, and the last-token scoring
that turns a patched KV cache into next-token logits and KL.

* ``prefill``         ToyTransformer.prefill          src/deltakv/model.py:141-172
                      (ToyBlock.forward / project_kv / attention / mlp, model.py:59-116;
                      causal mask model.py:138-139)
* ``logits_from_kv``  ToyTransformer.logits_from_kv   src/deltakv/model.py:229-253
                      (ToyBlock.attention/mlp/_repeat_kv, model.py:74-102; silu from
                      patches/analytic.py; RMSNorm model.py:48-56; tied lm_head)
* ``next_token_kl``   metrics.next_token_kl           src/deltakv/metrics.py:92-98
"""

from __future__ import annotations

import numpy as np

from oracle.exact import apply_rope, rmsnorm

F32 = np.float32


def _silu(x):
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def _softmax(x, axis=-1):
    m = x.max(axis=axis, keepdims=True)
    e = np.exp((x - m).astype(np.float64))
    return (e / e.sum(axis=axis, keepdims=True)).astype(F32)


def prefill(w: dict, token_ids: np.ndarray, *, n_layers: int, n_heads: int, n_kv: int, hd: int, eps: float,
            rope: tuple) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Full causal prefill of ``token_ids``: returns ``(last-position logits, k, v, h_in)``
    with ``k, v [L, seq, n_kv, hd]`` (K rotated) and ``h_in [L, seq, d]`` the residual
    stream entering each block (what the engine stores as the layer's activations)."""
    seq = token_ids.shape[0]
    x = w["embed_weight"][token_ids].astype(F32)
    pos = np.arange(seq)
    rep = n_heads // n_kv
    causal = np.triu(np.ones((seq, seq), bool), k=1)
    ks, vs, hs = [], [], []
    for i in range(n_layers):
        p = f"blocks_{i}_"
        hs.append(x.copy())
        xn = rmsnorm(x, w[p + "attn_norm_weight"], eps)
        q = apply_rope((xn @ w[p + "q_proj_weight"].T).reshape(seq, n_heads, hd), rope[0], rope[1], pos)
        k = apply_rope((xn @ w[p + "k_proj_weight"].T).reshape(seq, n_kv, hd), rope[0], rope[1], pos)
        v = (xn @ w[p + "v_proj_weight"].T).reshape(seq, n_kv, hd).astype(F32)
        ks.append(k)
        vs.append(v)
        kf = np.repeat(k, rep, axis=1) if rep > 1 else k
        vf = np.repeat(v, rep, axis=1) if rep > 1 else v
        ctx = np.empty((seq, n_heads, hd), F32)
        for h in range(n_heads):  # one head at a time bounds the [seq, seq] temporaries
            s_ = (q[:, h] @ kf[:, h].T).astype(F32) * F32(hd ** -0.5)
            s_[causal] = -np.inf
            ctx[:, h] = _softmax(s_) @ vf[:, h]
        x = x + ctx.reshape(seq, -1) @ w[p + "o_proj_weight"].T
        xm = rmsnorm(x, w[p + "mlp_norm_weight"], eps)
        x = (x + (_silu(xm @ w[p + "gate_proj_weight"].T) * (xm @ w[p + "up_proj_weight"].T))
             @ w[p + "down_proj_weight"].T).astype(F32)
    head = w.get("lm_head_weight", w["embed_weight"])
    logits = (rmsnorm(x[-1:], w["final_norm_weight"], eps) @ head.T).reshape(-1).astype(F32)
    return logits, np.stack(ks), np.stack(vs), np.stack(hs)


def logits_from_kv(w: dict, token_ids: np.ndarray, k: np.ndarray, v: np.ndarray, *, n_layers: int,
                   n_heads: int, n_kv: int, hd: int, eps: float, rope: tuple) -> np.ndarray:
    """Next-token logits at the last position given ``k, v [L, seq, n_kv, hd]``.

    ``w`` maps ``"embed_weight"``, ``"blocks_{i}_q_proj_weight"``, ... to arrays (the toy's
    state_dict with dots replaced by underscores)."""
    last = int(token_ids[-1])
    x = w["embed_weight"][last][None, :].astype(F32)
    pos = k.shape[1] - 1
    rep = n_heads // n_kv
    for i in range(n_layers):
        p = f"blocks_{i}_"
        xn = rmsnorm(x, w[p + "attn_norm_weight"], eps)
        q = (xn @ w[p + "q_proj_weight"].T).reshape(1, n_heads, hd)
        q = apply_rope(q, rope[0], rope[1], np.array([pos]))
        kf = np.repeat(k[i], rep, axis=1) if rep > 1 else k[i]
        vf = np.repeat(v[i], rep, axis=1) if rep > 1 else v[i]
        scores = np.einsum("qhd,khd->hqk", q, kf).astype(F32) * F32(hd ** -0.5)
        attn = _softmax(scores)
        ctx = np.einsum("hqk,khd->qhd", attn, vf).astype(F32).reshape(1, -1)
        x = x + ctx @ w[p + "o_proj_weight"].T
        xm = rmsnorm(x, w[p + "mlp_norm_weight"], eps)
        x = x + (_silu(xm @ w[p + "gate_proj_weight"].T) * (xm @ w[p + "up_proj_weight"].T)) @ w[p + "down_proj_weight"].T
    head = w.get("lm_head_weight", w["embed_weight"])
    return (rmsnorm(x, w["final_norm_weight"], eps) @ head.T).reshape(-1).astype(F32)


def next_token_kl(logits_p: np.ndarray, logits_q: np.ndarray) -> float:
    """KL(P || Q) in nats of the last-position distributions."""
    def log_softmax(z):
        z = z.astype(np.float64)
        m = z.max()
        return z - m - np.log(np.exp(z - m).sum())
    lp, lq = log_softmax(logits_p), log_softmax(logits_q)
    return float(max(0.0, (np.exp(lp) * (lp - lq)).sum()))


def weights_from_golden(g: dict) -> dict:
    return {k[2:]: v for k, v in g.items() if k.startswith("w_")}
