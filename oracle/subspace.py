"""Oracle of the subspace route (numpy fp32; TEST INFRASTRUCTURE ONLY).

* ``svd_basis``        subspace.svd_basis       src/deltakv/patches/subspace.py:37-42
* ``solve_codes``      subspace._solve_codes    src/deltakv/patches/subspace.py:21-34
* ``subspace_correct`` subspace.subspace_correct src/deltakv/patches/subspace.py:45-106
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def svd_basis(residual: np.ndarray, rank: int) -> np.ndarray:
    r = max(1, min(int(rank), residual.shape[0], residual.shape[1]))
    _, _, vh = np.linalg.svd(residual.astype(F32), full_matrices=False)
    return np.ascontiguousarray(vh[:r].T.astype(F32))


def solve_codes(residual: np.ndarray, basis: np.ndarray) -> np.ndarray:
    gram = basis.T @ basis
    eye = np.eye(gram.shape[0], dtype=gram.dtype)
    rhs = residual @ basis
    return np.linalg.solve(gram + F32(1e-6) * eye, rhs.T).T.astype(F32)


def subspace_correct(reused: np.ndarray, fresh: np.ndarray, probe_index, *, basis=None, rank: int = 8,
                     token_weights=None):
    """Returns ``(corrected [seq, n_kv, hd], subspace [d], orth_mu [d])`` in fp32."""
    seq, n_kv, hd = reused.shape
    idx = np.asarray(probe_index, dtype=np.int64).reshape(-1)
    rf = reused.reshape(seq, -1).astype(F32)
    ff = fresh.reshape(seq, -1).astype(F32)
    residual = ff - rf
    rp = residual[idx]
    d = rf.shape[-1]
    if basis is None:
        r_eff = min(rank, max(1, int(idx.size) - 1), d)
        basis = svd_basis(rp, r_eff) if rp.shape[0] >= 2 else None
    if basis is not None and basis.size and idx.size >= 1:
        if basis.shape[0] != d:
            raise ValueError(f"basis d={basis.shape[0]} != kv d={d}")
        basis = basis.astype(F32)
        codes = solve_codes(residual, basis)
        fitted = codes @ basis.T
        subspace = codes.mean(axis=0) @ basis.T
        orth_mu = (rp - fitted[idx]).mean(axis=0)
        structured = True
        field = fitted
    else:
        subspace = np.zeros(d, F32)
        orth_mu = rp.mean(axis=0) if rp.size else np.zeros(d, F32)
        structured = False
        field = np.zeros((seq, d), F32)
    if token_weights is None:
        dist = np.linalg.norm(residual, axis=-1)
        scale = max(float(dist.mean()), 1e-8) if dist.size else 1e-8
        w = np.minimum(dist / F32(scale), 1.0).astype(F32)
    else:
        w = np.asarray(token_weights, F32)
    corr = rf + field + w[:, None] * orth_mu[None, :]
    if not structured:
        corr = rf + w[:, None] * orth_mu[None, :]
    corr[idx] = ff[idx]
    return corr.reshape(seq, n_kv, hd).astype(F32), np.asarray(subspace, F32), np.asarray(orth_mu, F32)
