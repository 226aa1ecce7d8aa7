"""Seeded SmolLM2-135M-shaped decoder weights and LoRA delta, shared by the golden generator
(which loads them into the reference's ToyTransformer) and the tests (which feed them to the
oracle and the kernels), so both sides see identical numbers without a large fixture.

Shape: d=576, 9 query / 3 KV heads of 64, SwiGLU 1536, vocab 49152, RMSNorm eps 1e-6, RoPE
base 1e4, tied embeddings — reduced to ``N_LAYERS`` layers (the full model has 30), because
the fp32 oracle prefill of 30 layers x 2048 tokens would not fit a test's time budget.
Linear weights and the embedding N(0, 0.02^2) as ToyTransformer._init_weights draws them
(src/deltakv/model.py:135-139); norm weights 1 + N(0, 0.05^2) so the folded RMSNorm weight
is exercised.  The delta: rank-8 LoRA on q/k/v/o of every layer, A ~ N(0, 1/d_in),
B ~ N(0, 1), scaled so ||s B A||_F = 0.01 ||W||_F.
"""

from __future__ import annotations

import math

import numpy as np

N_LAYERS = 4
D, N_HEADS, N_KV, HD, D_FF, VOCAB = 576, 9, 3, 64, 1536, 49152
EPS, ROPE_BASE, SEQ, RANK = 1e-6, 10000.0, 2048, 8
PROJ = {"q_proj": (D, N_HEADS * HD), "k_proj": (D, N_KV * HD), "v_proj": (D, N_KV * HD), "o_proj": (N_HEADS * HD, D)}


def weights(seed: int = 0) -> dict[str, np.ndarray]:
    """Oracle-named fp32 weights (``state_dict`` keys with dots replaced by underscores)."""
    rng = np.random.default_rng(seed)
    nrm = lambda *s: (0.02 * rng.standard_normal(s)).astype(np.float32)
    w = {"embed_weight": nrm(VOCAB, D)}
    for i in range(N_LAYERS):
        p = f"blocks_{i}_"
        w[p + "attn_norm_weight"] = (1 + 0.05 * rng.standard_normal(D)).astype(np.float32)
        for name, (fin, fout) in PROJ.items():
            w[p + name + "_weight"] = nrm(fout, fin)
        w[p + "mlp_norm_weight"] = (1 + 0.05 * rng.standard_normal(D)).astype(np.float32)
        w[p + "gate_proj_weight"] = nrm(D_FF, D)
        w[p + "up_proj_weight"] = nrm(D_FF, D)
        w[p + "down_proj_weight"] = nrm(D, D_FF)
    w["final_norm_weight"] = (1 + 0.05 * rng.standard_normal(D)).astype(np.float32)
    return w


def tokens(seed: int = 1) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, VOCAB, size=SEQ).astype(np.int64)


def delta(w: dict[str, np.ndarray], seed: int = 2) -> dict[int, dict[str, tuple[np.ndarray, np.ndarray, float]]]:
    """``{layer: {proj: (A [r, d_in], B [d_out, r], scale)}}``."""
    rng = np.random.default_rng(seed)
    out = {}
    for i in range(N_LAYERS):
        out[i] = {}
        for name, (fin, fout) in PROJ.items():
            A = (rng.standard_normal((RANK, fin)) / math.sqrt(fin)).astype(np.float32)
            B = rng.standard_normal((fout, RANK)).astype(np.float32)
            W = w[f"blocks_{i}_{name}_weight"]
            s = float(0.01 * np.linalg.norm(W) / np.linalg.norm(B.astype(np.float64) @ A.astype(np.float64)))
            out[i][name] = (A, B, s)
    return out


def merged(w: dict[str, np.ndarray], dl: dict) -> dict[str, np.ndarray]:
    """W + s B A for every factored projection (ToyTransformer.apply_delta, model.py:255-274)."""
    out = dict(w)
    for i, projs in dl.items():
        for name, (A, B, s) in projs.items():
            key = f"blocks_{i}_{name}_weight"
            out[key] = (w[key] + np.float32(s) * (B @ A)).astype(np.float32)
    return out


def dense_delta(w: dict[str, np.ndarray], seed: int = 3, rel: float = 0.02) -> dict[int, dict[str, np.ndarray]]:
    """A full-rank dW on k_proj and v_proj of every layer (an RL step's delta), Gaussian with
    ||dW||_F = rel ||W||_F, rounded to bf16 values (the dense route's operand type)."""
    rng = np.random.default_rng(seed)
    out = {}
    for i in range(N_LAYERS):
        out[i] = {}
        for name in ("k_proj", "v_proj"):
            W = w[f"blocks_{i}_{name}_weight"]
            dw = rng.standard_normal(W.shape).astype(np.float32)
            dw *= np.float32(rel * np.linalg.norm(W) / np.linalg.norm(dw))
            out[i][name] = _to_bf16(dw)
    return out


def merged_dense(w: dict[str, np.ndarray], dd: dict) -> dict[str, np.ndarray]:
    out = dict(w)
    for i, projs in dd.items():
        for name, dw in projs.items():
            key = f"blocks_{i}_{name}_weight"
            out[key] = (w[key] + dw).astype(np.float32)
    return out


def _to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) & np.uint32(0xFFFF0000)).view(np.float32)
    return r.astype(np.float32)
