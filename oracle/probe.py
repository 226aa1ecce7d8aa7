"""Oracle of probe scoring/selection, the residual gate, the probe route per layer and the
STRICT-hit replay (numpy; TEST INFRASTRUCTURE ONLY).

* ``lora_activation_scores`` exact.lora_activation_scores  src/deltakv/patches/exact.py:111-115
* ``weight_axis_scores``     probe.weight_axis_scores      src/deltakv/patches/probe.py:30-47
* ``select_probes``          probe.select_probes           src/deltakv/patches/probe.py:14-27
* ``residual_gate``          probe.residual_gate           src/deltakv/patches/probe.py:85-109
* ``apply_probe_to_cache``   probe.apply_probe_to_cache    src/deltakv/patches/probe.py:112-165
* ``replay``                 engine._replay + compose.apply_layer_patches
                             src/deltakv/engine.py:205-210, src/deltakv/patches/compose.py:29-34
"""

from __future__ import annotations

import numpy as np

from oracle.subspace import subspace_correct

F32 = np.float32


def lora_activation_scores(x: np.ndarray, a: np.ndarray, scale: float) -> np.ndarray:
    codes = (F32(scale) * (np.asarray(x, F32) @ np.asarray(a, F32).T)).astype(F32)
    return np.linalg.norm(codes, axis=-1).astype(F32)


def weight_axis_scores(x: np.ndarray, factors: list) -> np.ndarray:
    """``factors`` = the (A, scale) pairs of the layer's projections."""
    acc = np.zeros(x.shape[0], F32)
    for a, s in factors:
        if a.shape[1] == x.shape[-1]:
            acc = acc + lora_activation_scores(x, a, s)
    return np.ones(x.shape[0], F32) if float(acc.max()) <= 0 else acc


def select_probes(scores: np.ndarray, ratio: float, min_tokens: int = 4, max_ratio: float = 0.5) -> np.ndarray:
    n = int(scores.size)
    b = int(max(min_tokens, round(ratio * n)))
    b = min(b, max(1, int(max_ratio * n)), n)
    top = np.argsort(-scores, kind="stable")[:b]
    if 0 not in top.tolist():
        top = np.concatenate([[0], top[:-1]])
    return np.unique(np.sort(top))


def residual_gate(reused, corrected, fresh_probe, probe_index, threshold: float, max_ratio: float) -> np.ndarray:
    seq = reused.shape[0]
    est = np.linalg.norm((corrected - reused).reshape(seq, -1), axis=-1)
    idx = np.asarray(probe_index, np.int64)
    probe_scale = np.linalg.norm((fresh_probe[idx] - reused[idx]).reshape(idx.size, -1), axis=-1)
    scale = max(float(probe_scale.mean()), 1e-8)
    relative = est / scale
    extra = np.nonzero(relative > threshold)[0]
    cap = max(0, int(max_ratio * seq) - int(idx.size))
    if extra.size > cap:
        extra = extra[np.argsort(-relative[extra], kind="stable")[:cap]]
    return extra


def apply_probe_to_cache(k, v, fresh: dict, probe_index, blend_threshold, blend_max_ratio, *, v_bases: dict,
                         k_ranks: dict, subspace_rank: int = 8, probe_layers=None):
    """``k``/``v`` ``[L, seq, n_kv, hd]``; returns (k_out, v_out, extra indices)."""
    k_out, v_out = k.copy(), v.copy()
    extra_all = []
    for l, (fk, fv) in fresh.items():
        rk, rv = k_out[l].copy(), v_out[l].copy()
        k_c, _, _ = subspace_correct(rk, fk, probe_index, basis=None, rank=k_ranks.get(l, subspace_rank))
        v_c, _, _ = subspace_correct(rv, fv, probe_index, basis=v_bases.get(l), rank=subspace_rank)
        if probe_layers is None or l in probe_layers:
            extra = residual_gate(rk, k_c, fk, probe_index, blend_threshold, blend_max_ratio)
            if extra.size:
                k_c[extra] = fk[extra]
                v_c[extra] = fv[extra]
                extra_all.append(extra)
        k_out[l], v_out[l] = k_c, v_c
    extra = np.unique(np.concatenate(extra_all)) if extra_all else np.zeros(0, np.int64)
    return k_out, v_out, extra


def replay(base_k, base_v, chain: list) -> tuple[np.ndarray, np.ndarray]:
    """``chain`` = stages of {layer: dict(k_codes, k_basis, v_codes, v_basis, k_dense, v_dense)}."""
    k, v = base_k.astype(F32).copy(), base_v.astype(F32).copy()
    n_kv, hd = k.shape[2], k.shape[3]
    for stage in chain:
        for l, p in stage.items():
            for dst, nm in ((k, "k"), (v, "v")):
                dense = p.get(f"{nm}_dense")
                if dense is None:
                    dense = (p[f"{nm}_codes"].astype(F32) @ p[f"{nm}_basis"].astype(F32).T).reshape(-1, n_kv, hd)
                dst[l] = dst[l] + dense
    return k, v
