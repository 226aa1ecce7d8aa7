"""Oracle of the per-layer measured patch error and KV comparison (numpy; TEST
INFRASTRUCTURE ONLY).

Restates ``measured_error`` (src/deltakv/patches/compose.py:147-163): per layer
``(||K_p - K_f|| + ||V_p - V_f||) / (||K_f|| + ||V_f|| + 1e-8)``, and its maximum; and
``compare_kv`` (src/deltakv/metrics.py:52-81): per layer and projection
``||p - f|| / (||f|| + 1e-8)`` and the cosine ``p.f / max(||p|| ||f||, 1e-8)``, then the
max / mean of the per-layer worse relative L2 and the min of the per-layer worse cosine.
"""

from __future__ import annotations

import numpy as np


def measured_error(pk: np.ndarray, pv: np.ndarray, fk: np.ndarray, fv: np.ndarray) -> tuple[float, list[float]]:
    per = []
    for l in range(pk.shape[0]):
        a = lambda x: np.asarray(x, np.float64)
        num = np.linalg.norm(a(pk[l]) - a(fk[l])) + np.linalg.norm(a(pv[l]) - a(fv[l]))
        den = np.linalg.norm(a(fk[l])) + np.linalg.norm(a(fv[l])) + 1e-8
        per.append(float(num / den))
    return (max(per) if per else 0.0), per


def compare_kv(pk: np.ndarray, pv: np.ndarray, fk: np.ndarray, fv: np.ndarray):
    """``(per-layer [n_layers, 4] (rel_k, rel_v, cos_k, cos_v), max_rel, mean_rel, min_cos)``."""
    a = lambda x: np.asarray(x, np.float64).ravel()
    rows = []
    for l in range(pk.shape[0]):
        r = []
        for p, f in ((pk[l], fk[l]), (pv[l], fv[l])):
            r.append(np.linalg.norm(a(p) - a(f)) / (np.linalg.norm(a(f)) + 1e-8))
        for p, f in ((pk[l], fk[l]), (pv[l], fv[l])):
            r.append(float(a(p) @ a(f)) / max(np.linalg.norm(a(p)) * np.linalg.norm(a(f)), 1e-8))
        rows.append(r)
    rows = np.array(rows, np.float64).reshape(-1, 4)
    rels = np.maximum(rows[:, 0], rows[:, 1]) if len(rows) else np.zeros(0)
    cos = np.minimum(rows[:, 2], rows[:, 3]) if len(rows) else np.zeros(0)
    return (rows, float(rels.max()) if len(rels) else 0.0, float(rels.mean()) if len(rels) else 0.0,
            float(cos.min()) if len(cos) else 1.0)

