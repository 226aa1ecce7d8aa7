"""dkv_split_gemm_batched (the K basis' thin products) against an fp64 product.

Tolerance: rel-L2 2e-5 per batch element.  Every operand is split into two bf16 terms and the
three leading cross products are accumulated in fp32, so a product is within ~1e-5 relative of
the fp32 one; the subspace iteration built on it is held to the exact basis in
tests/test_topr_basis.py.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200 import _lib as L
from deltakv_b200 import ops
from deltakv_b200.subspace import thin_mm

pytestmark = pytest.mark.gpu


def _ref(a, b, trans):
    a64, b64 = a.double(), b.double()
    return torch.matmul(a64.transpose(1, 2) if trans else a64, b64)


@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("n", [16, 48, 96])
@pytest.mark.parametrize("m,k", [(777, 264), (64, 4), (1024, 3277), (5, 1000)])
def test_split_gemm_matches_fp64(cuda, trans, n, m, k):
    if trans and m % 4:
        pytest.skip("m % 4 with trans_a")
    if not trans and k % 4:
        pytest.skip("k % 4")
    gen = torch.Generator(device=cuda).manual_seed(m * 7 + k + n)
    bt = 3
    a = torch.randn(bt, k, m, generator=gen, device=cuda) if trans else torch.randn(bt, m, k, generator=gen, device=cuda)
    a *= torch.logspace(-2, 2, a.shape[-1], device=cuda)  # columns over four decades
    b = torch.randn(bt, k, n, generator=gen, device=cuda)
    c = torch.full((bt, m, n), float("nan"), device=cuda)
    rc = L.lib().dkv_split_gemm_batched(a.data_ptr(), a.stride(0), a.stride(1), int(trans), b.data_ptr(), b.stride(0),
                                        b.stride(1), c.data_ptr(), c.stride(0), c.stride(1), bt, m, n, k,
                                        ops.stream_ptr())
    assert rc == L.DKV_OK
    ref = _ref(a, b, trans)
    for i in range(bt):
        err = float((c[i].double() - ref[i]).norm() / ref[i].norm())
        assert err < 2e-5, (i, err)


def test_split_gemm_strided_batches_and_padding(cuda):
    # batch strides and leading dimensions wider than the rows; zero columns past n stay zero,
    # so a padded result feeds the next product directly (Y = X Q, then Z = X^T Y)
    gen = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(2, 500, 136, generator=gen, device=cuda)[:, :, :128]  # lda 136
    q = torch.zeros(2, 128, 32, device=cuda)
    q[:, :, :20] = torch.randn(2, 128, 20, generator=gen, device=cuda)
    y = thin_mm(x, q)
    assert y.shape == (2, 500, 32) and torch.count_nonzero(y[:, :, 20:]) == 0
    z = thin_mm(x, y, trans_a=True)
    ref = x.double().transpose(1, 2) @ (x.double() @ q.double())
    assert float((z.double() - ref).norm() / ref.norm()) < 2e-5


def test_thin_mm_pads_and_falls_back(cuda):
    gen = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(2, 300, 256, generator=gen, device=cuda)
    q = torch.randn(2, 256, 24, generator=gen, device=cuda)
    y = thin_mm(x, q)  # 24 columns -> 32, zero padded
    assert y.shape == (2, 300, 32)
    ref = x.double() @ q.double()
    assert float((y[:, :, :24].double() - ref).norm() / ref.norm()) < 2e-5
    assert torch.count_nonzero(y[:, :, 24:]) == 0
    wide = torch.randn(2, 256, 100, generator=gen, device=cuda)  # wider than the kernel takes
    np.testing.assert_allclose(thin_mm(x, wide).cpu().numpy(), torch.matmul(x, wide).cpu().numpy(), rtol=1e-5,
                               atol=1e-4)
