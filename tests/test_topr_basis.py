"""The batched top-r subspace (K-basis of the int4 subspace route) against the exact SVD.

``topr_basis`` must span the same subspace as the reference's ``svd_basis`` (a full SVD);
the least-squares correction depends on the basis only through that column space, so the
check is on the orthogonal projectors.  Runs on CPU torch.
"""

from __future__ import annotations

import torch

from deltakv_b200.subspace import svd_basis, topr_basis


def _proj_diff(a, b):
    pa, pb = a @ a.T, b @ b.T
    return float((pa - pb).norm() / pa.norm())


def test_topr_basis_matches_svd_on_low_rank_plus_noise():
    g = torch.Generator().manual_seed(0)
    for m, d, r in ((400, 128, 8), (300, 256, 16), (200, 64, 4)):
        x = torch.randn(m, r, generator=g) @ torch.randn(r, d, generator=g) + 0.05 * torch.randn(m, d, generator=g)
        assert _proj_diff(svd_basis(x, r), topr_basis(x, r)) < 1e-4


def test_topr_basis_batched_and_orthonormal():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3, 200, 6, generator=g) @ torch.randn(3, 6, 96, generator=g) + 0.01 * torch.randn(3, 200, 96, generator=g)
    b = topr_basis(x, 6)
    assert b.shape == (3, 96, 6)
    for i in range(3):
        assert torch.allclose(b[i].T @ b[i], torch.eye(6), atol=1e-4)
        assert _proj_diff(svd_basis(x[i], 6), b[i]) < 1e-4


def test_topr_basis_falls_back_to_svd_without_a_gap():
    # isotropic noise has no spectral gap: the iteration cannot settle, the exact SVD is used
    g = torch.Generator().manual_seed(2)
    x = torch.randn(500, 256, generator=g)
    assert _proj_diff(svd_basis(x, 8), topr_basis(x, 8)) < 1e-5
