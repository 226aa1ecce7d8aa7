"""Oracle of the per-layer measured patch error (numpy; TEST INFRASTRUCTURE ONLY).

Restates ``measured_error`` (src/deltakv/patches/compose.py:147-163): per layer
``(||K_p - K_f|| + ||V_p - V_f||) / (||K_f|| + ||V_f|| + 1e-8)``, and its maximum.
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
