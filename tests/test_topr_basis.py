"""The batched top-r subspace (K-basis of the int4 subspace route) against the exact SVD, and
its device eigensolver (``dkv_sym_eig_batched``) against LAPACK.

``topr_basis`` must span the same subspace as the reference's ``svd_basis`` (a full SVD);
the least-squares correction depends on the basis only through that column space, so the
check is on the orthogonal projectors: relative Frobenius difference below 1e-5 from an fp64
SVD (the fp32 device SVD itself is only good to ~5e-4 at 1500 x 1024, rank 64), also where the
exact path (fp64 Gram matrix + eigensolver) must take over.  The eigensolver: eigenvalues
within 1e-10 of the largest magnitude, eigenvectors orthonormal to 1e-10 and
A V = V diag(ev) to 1e-9 (fp64).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200.subspace import gram_basis, sym_eig, topr_basis

pytestmark = pytest.mark.gpu


def _proj_diff(a, b):
    a, b = a.double(), b.double()
    pa, pb = a @ a.T, b @ b.T
    return float((pa - pb).norm() / pa.norm())


def _truth(x, r):
    return torch.linalg.svd(x.double(), full_matrices=False)[2][:r].T


def test_topr_basis_matches_svd_on_low_rank_plus_noise(cuda):
    g = torch.Generator().manual_seed(0)
    for m, d, r in ((400, 128, 8), (300, 256, 16), (200, 64, 4), (1500, 1024, 64)):
        x = torch.randn(m, r, generator=g) @ torch.randn(r, d, generator=g) + 0.05 * torch.randn(m, d, generator=g)
        x = x.to(cuda)
        assert _proj_diff(_truth(x, r), topr_basis(x, r)) < 1e-5


def test_topr_basis_batched_and_orthonormal(cuda):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3, 200, 6, generator=g) @ torch.randn(3, 6, 96, generator=g) + 0.01 * torch.randn(3, 200, 96, generator=g)
    x = x.to(cuda)
    b = topr_basis(x, 6)
    assert b.shape == (3, 96, 6)
    eye = torch.eye(6, device=cuda)
    for i in range(3):
        assert torch.allclose(b[i].T @ b[i], eye, atol=1e-4)
        assert _proj_diff(_truth(x[i], 6), b[i]) < 1e-5


def test_topr_basis_falls_back_without_a_gap(cuda, monkeypatch):
    # isotropic noise has no spectral gap: the iteration cannot settle, the exact path is used
    # right after the first estimate (the extrapolated one cannot reach the tolerance)
    import deltakv_b200.subspace as S

    calls = []
    monkeypatch.setattr(S, "gram_basis", lambda x, r: calls.append(x.shape[0]) or gram_basis(x, r))
    g = torch.Generator().manual_seed(2)
    x = torch.randn(500, 256, generator=g).to(cuda)
    b = S.topr_basis(x, 8)
    assert calls == [1]
    # a gapless spectrum: compare the projectors of the exact paths (fp64 SVD vs fp64 Gram)
    assert _proj_diff(_truth(x, 8), b) < 1e-5


def test_topr_basis_iterates_further_before_falling_back(cuda, monkeypatch):
    # eigenvalue ratio 1e-2 past the rank: two iterations estimate 1e-4 (too coarse), the
    # third 1e-6 — settled by iterating, without the SVD
    import deltakv_b200.subspace as S

    calls = []
    monkeypatch.setattr(S, "gram_basis", lambda x, r: calls.append(1) or gram_basis(x, r))
    g = torch.Generator().manual_seed(4)
    m, d, r = 600, 256, 8
    u, _ = torch.linalg.qr(torch.randn(m, d, generator=g, dtype=torch.float64))
    v, _ = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64))
    sv = torch.cat([torch.linspace(2.0, 1.0, r, dtype=torch.float64), 0.1 * torch.linspace(1.0, 0.5, d - r, dtype=torch.float64)])
    x = ((u * sv) @ v.T).float().to(cuda)
    b = S.topr_basis(torch.stack([x, x]), r)
    assert not calls
    assert _proj_diff(v[:, :r].float().to(cuda), b[0]) < 1e-5
    assert _proj_diff(v[:, :r].float().to(cuda), b[1]) < 1e-5
    one = S.topr_basis(x, r, iters=2)  # capped at two: the estimate fails, the exact path is used
    assert calls and _proj_diff(v[:, :r].float().to(cuda), one) < 1e-5


def test_topr_basis_few_rows_uses_the_exact_path(cuda):
    # m <= rank + oversample: the fp64 Gram eigensolver directly
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 10, 64, generator=g).to(cuda)
    b = topr_basis(x, 4)
    for i in range(2):
        assert _proj_diff(_truth(x[i], 4), b[i]) < 1e-5


def _check_eig(a, ev, vec):
    for i in range(a.shape[0]):
        ref = np.linalg.eigvalsh(a[i])[::-1]
        scale = max(1.0, float(np.abs(ref).max()))
        assert np.abs(ev[i] - ref).max() <= 1e-10 * scale
        v = vec[i]
        assert np.abs(v.T @ v - np.eye(v.shape[1])).max() <= 1e-10
        assert np.abs(a[i] @ v - v * ev[i][None, :]).max() <= 1e-9 * scale
        assert np.all(np.diff(ev[i]) <= 0)


@pytest.mark.parametrize("k", [1, 2, 7, 16, 33, 72, 96])
def test_sym_eig_matches_lapack(cuda, k):
    rng = np.random.default_rng(k)
    a = rng.standard_normal((5, k, k))
    a = a + a.transpose(0, 2, 1)
    a[1] = np.diag(rng.standard_normal(k))  # already diagonal
    ev, vec, info = sym_eig(torch.from_numpy(a).to(cuda))
    assert info.cpu().tolist() == [0] * 5
    _check_eig(a, ev.cpu().numpy(), vec.cpu().numpy())


def test_sym_eig_graded_and_degenerate_spectra(cuda):
    # the Rayleigh-Ritz matrices of the K basis: eigenvalues spread over many decades, and
    # exactly repeated eigenvalues (zero matrix, identity, a rank-deficient Gram)
    rng = np.random.default_rng(7)
    k = 72
    q, _ = np.linalg.qr(rng.standard_normal((k, k)))
    graded = (q * np.logspace(6, -8, k)[None, :]) @ q.T
    low = rng.standard_normal((k, 5))
    mats = np.stack([graded, np.zeros((k, k)), np.eye(k) * 3.0, low @ low.T])
    ev, vec, info = sym_eig(torch.from_numpy(mats).to(cuda))
    assert info.cpu().tolist() == [0, 0, 0, 0]
    _check_eig(mats, ev.cpu().numpy(), vec.cpu().numpy())


def test_sym_eig_reports_non_finite_input(cuda):
    a = np.eye(8)[None].repeat(2, axis=0)
    a[1, 2, 3] = np.nan
    ev, vec, info = sym_eig(torch.from_numpy(a).to(cuda))
    assert info.cpu().tolist() == [0, 2]
    assert np.allclose(ev.cpu().numpy()[0], 1.0)
