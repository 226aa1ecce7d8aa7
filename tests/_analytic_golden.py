"""Unpacks tests/golden/analytic.npz (the reference's analytic route on a GQA toy) for the oracle
and GPU tests."""

from __future__ import annotations

import numpy as np

from tests.conftest import golden

PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def load():
    g = golden("analytic")
    L = int(g["n_layers"])
    weights = []
    for l in range(L):
        w = {p: g[f"w_blocks_{l}_{p}_proj_weight"] for p in PROJ}
        w["attn_norm"] = g[f"w_blocks_{l}_attn_norm_weight"]
        w["mlp_norm"] = g[f"w_blocks_{l}_mlp_norm_weight"]
        weights.append(w)
    layers = {}
    for l in range(L):
        facs = {p: (g[f"lora_{l}_{p}_A"], g[f"lora_{l}_{p}_B"], float(g[f"lora_{l}_{p}_scale"]))
                for p in PROJ if f"lora_{l}_{p}_A" in g}
        if facs:
            layers[l] = facs
    cfg = dict(n_heads=int(g["n_heads"]), n_kv=int(g["n_kv"]), hd=int(g["hd"]), d_model=int(g["d_model"]),
               eps=float(g["eps"]), rope_base=float(g["rope_base"]), rope_max=int(g["rope_max"]),
               hidden_stride=int(g["hidden_stride"]), propagator_rank=int(g["propagator_rank"]))
    return g, weights, layers, cfg


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))
