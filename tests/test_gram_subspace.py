"""The fused subspace iteration on an fp64 Gram matrix (``dkv_gram_subspace_iterate``) against
numpy, and :func:`gram_topr_basis` — the analytic route's rank truncation basis — against the
exact top-r eigen-subspace.

One step must be Cholesky QR of G Q to fp64 rounding (1e-9 of the largest entry; Q^T Q = I to
1e-10; the Rayleigh quotient Q^T G Q to 1e-10); several steps must span numpy's subspace
(projector difference 1e-8).  ``gram_topr_basis`` on a spectrum shaped like the propagated
ΔX (singular values 1 % apart at the cut): ||x (P - P_exact)||_F / ||x||_F <= 1e-6 without the
exact path; small / rank-deficient / degenerate inputs take the exact paths.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200 import _lib as L
from deltakv_b200 import ops

pytestmark = pytest.mark.gpu


def _iterate(g: np.ndarray, q0: np.ndarray, iters: int, cuda):
    d, k = q0.shape
    G = torch.from_numpy(np.ascontiguousarray(g)).to(cuda)
    Q = torch.from_numpy(np.ascontiguousarray(q0)).to(cuda)
    y = torch.empty(d, k, dtype=torch.float64, device=cuda)
    w = torch.empty(2, k, k, dtype=torch.float64, device=cuda)
    t = torch.empty(k, k, dtype=torch.float64, device=cuda)
    st = torch.empty(1, dtype=torch.int32, device=cuda)
    rc = L.lib().dkv_gram_subspace_iterate(G.data_ptr(), d, Q.data_ptr(), k, iters, y.data_ptr(), w.data_ptr(),
                                           t.data_ptr(), st.data_ptr(), ops.stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    return Q.cpu().numpy(), t.cpu().numpy(), y.cpu().numpy(), int(st.item())


def _gram(rng, m, d, decades=2.0):
    x = rng.standard_normal((m, d)) * np.logspace(0, -decades, d)
    g = x.T @ x
    return 0.5 * (g + g.T)


def _cholqr(y):
    r = np.linalg.cholesky(y.T @ y).T
    return np.linalg.solve(r.T, y.T).T


def test_one_step_is_cholesky_qr(cuda):
    rng = np.random.default_rng(0)
    d, k = 200, 40
    g = _gram(rng, 500, d)
    q0 = np.linalg.qr(rng.standard_normal((d, k)))[0]
    q, t, y, st = _iterate(g, q0, 1, cuda)
    assert st == 0
    want = _cholqr(g @ q0)
    assert np.abs(q - want).max() <= 1e-9 * np.abs(want).max()
    assert np.abs(q.T @ q - np.eye(k)).max() <= 1e-10
    rq = q.T @ g @ q
    assert np.abs(t - rq).max() <= 1e-10 * np.abs(rq).max()
    assert np.abs(y - g @ q).max() <= 1e-10 * np.abs(g @ q).max()


@pytest.mark.parametrize("d,k,iters", [(13, 5, 3), (96, 96, 2), (300, 72, 10), (577, 96, 6)])
def test_iterations_span_numpys_subspace(cuda, d, k, iters):
    rng = np.random.default_rng(d + k)
    g = _gram(rng, max(2 * d, 50), d, decades=1.0)
    q0 = rng.standard_normal((d, k))
    q, t, _, st = _iterate(g, q0, iters, cuda)
    assert st == 0
    want = q0
    for _ in range(iters):
        want = _cholqr(g @ want)
    assert np.abs(q @ q.T - want @ want.T).max() <= 1e-8
    assert np.abs(q.T @ q - np.eye(k)).max() <= 1e-9


def test_zero_steps_give_the_rayleigh_quotient_of_the_start(cuda):
    rng = np.random.default_rng(5)
    d, k = 150, 24
    g = _gram(rng, 300, d)
    q0 = np.linalg.qr(rng.standard_normal((d, k)))[0]
    q, t, _, st = _iterate(g, q0, 0, cuda)
    assert st == 0 and np.array_equal(q, q0)
    assert np.abs(t - q0.T @ g @ q0).max() <= 1e-10 * np.abs(t).max()


def test_a_block_that_lost_rank_is_flagged(cuda):
    rng = np.random.default_rng(6)
    x = rng.standard_normal((10, 100))  # G has rank 10 < k
    g = x.T @ x
    _, _, _, st = _iterate(0.5 * (g + g.T), rng.standard_normal((100, 32)), 1, cuda)
    assert st == 1


def test_invalid_arguments_are_rejected(cuda):
    z = torch.zeros(16, dtype=torch.float64, device=cuda)
    p = z.data_ptr()
    lib = L.lib()
    assert lib.dkv_gram_subspace_iterate(p, 8, p, 97, 1, p, p, p, p, ops.stream_ptr()) == L.DKV_ERR_INVALID_ARGUMENT
    assert lib.dkv_gram_subspace_iterate(p, 4, p, 5, 1, p, p, p, p, ops.stream_ptr()) == L.DKV_ERR_INVALID_ARGUMENT
    assert lib.dkv_gram_subspace_iterate(p, 8, p, 4, -1, p, p, p, p, ops.stream_ptr()) == L.DKV_ERR_INVALID_ARGUMENT


# singular values of the analytic route's propagated dX (SmolLM2-135M shape, 2048 tokens)
# at indices 0, 8, 16, 32, 48, 60, 63, 64, 65, 72, 80, 96, 128, 575
_PROFILE_AT = [0, 8, 16, 32, 48, 60, 63, 64, 65, 72, 80, 96, 128, 575]
_PROFILE = [1.0, 0.15, 0.09, 0.05, 0.037, 0.032, 0.0301, 0.0299, 0.0297, 0.026, 0.022, 0.017, 0.013, 0.004]


def _with_spectrum(m, d, s, seed):
    rng = np.random.default_rng(seed)
    u = np.linalg.qr(rng.standard_normal((m, d)))[0]
    v = np.linalg.qr(rng.standard_normal((d, d)))[0]
    return ((u * s) @ v.T).astype(np.float32)


def _exact_projector(x, r):
    g = x.astype(np.float64).T @ x.astype(np.float64)
    _, vec = np.linalg.eigh(g)
    v = vec[:, -r:]
    return v @ v.T


def _trunc_err(x, basis, r):
    x64 = x.astype(np.float64)
    b = basis.astype(np.float64)
    return np.linalg.norm(x64 @ (b @ b.T - _exact_projector(x, r))) / np.linalg.norm(x64)


def test_gram_topr_basis_on_a_gapless_spectrum(cuda, monkeypatch):
    import deltakv_b200.subspace as S

    exact_calls = []
    orig = S._eigh_top
    monkeypatch.setattr(S, "_eigh_top", lambda c, r: exact_calls.append(1) or orig(c, r))
    d, r = 576, 64
    s = np.interp(np.arange(d), _PROFILE_AT, _PROFILE)
    x = _with_spectrum(2048, d, s, 11)
    b = S.gram_topr_basis(torch.from_numpy(x).to(cuda), r).cpu().numpy()
    assert not exact_calls
    assert b.shape == (d, r)
    assert np.abs(b.T.astype(np.float64) @ b - np.eye(r)).max() <= 1e-6
    assert _trunc_err(x, b, r) <= 1e-6


def test_gram_topr_basis_small_and_rank_deficient_inputs(cuda):
    from deltakv_b200.subspace import gram_topr_basis

    rng = np.random.default_rng(12)
    for m, d, r in ((300, 64, 8), (50, 200, 16), (2000, 97, 40)):  # d <= 96: Jacobi on G; m < k: exact; d = 97: iteration
        x = (rng.standard_normal((m, d)) * np.logspace(0, -1.5, d)).astype(np.float32)
        b = gram_topr_basis(torch.from_numpy(x).to(cuda), r).cpu().numpy()
        assert b.shape == (d, r)
        assert _trunc_err(x, b, r) <= 1e-6


def test_gram_topr_basis_degenerate_and_zero_inputs(cuda):
    from deltakv_b200.subspace import gram_topr_basis

    d, r = 300, 32
    s = np.linspace(1.0, 0.1, d)
    s[r - 4: r + 4] = 0.5  # exactly repeated singular values across the cut
    x = _with_spectrum(600, d, s, 13)
    b = gram_topr_basis(torch.from_numpy(x).to(cuda), r).cpu().numpy().astype(np.float64)
    x64 = x.astype(np.float64)
    # any basis of a top-r subspace is optimal: the truncation error is the Eckart-Young one
    best = np.sqrt((np.linalg.svd(x64, compute_uv=False)[r:] ** 2).sum())
    assert abs(np.linalg.norm(x64 - x64 @ b @ b.T) - best) <= 1e-5 * best
    z = gram_topr_basis(torch.zeros(400, 200, device=cuda), 16)
    assert z.shape == (200, 16) and torch.isfinite(z).all()
