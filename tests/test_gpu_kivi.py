"""KIVI int4 kernels on the GPU: bit-exact against the oracle's restatement of the format."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200 import kivi as K
from oracle import kivi as OK

pytestmark = pytest.mark.gpu


def _np(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("mode", ["k", "v"])
@pytest.mark.parametrize("n,d,dtype", [(77, 64, torch.float32), (256, 1024, torch.bfloat16), (33, 96, torch.float16),
                                       (1, 32, torch.float32)])
def test_quantize_dequantize_bit_exact(cuda, mode, n, d, dtype):
    gen = torch.Generator().manual_seed(n * d)
    x = (torch.randn(n, d, generator=gen) * 2 + 0.3).to(dtype)
    q = K.quantize(x.to(cuda), mode)
    c, s, z = OK.quantize(x.float().numpy(), mode)
    assert np.array_equal(_np(q.codes), c)
    assert np.array_equal(_np(q.scale).view(np.uint16), s.view(np.uint16))
    assert np.array_equal(_np(q.zero).view(np.uint16), z.view(np.uint16))
    deq = K.dequantize(q, torch.float32)
    assert np.array_equal(_np(deq), OK.dequantize(c, s, z, mode))


@pytest.mark.parametrize("mode", ["k", "v"])
@pytest.mark.parametrize("inplace", [False, True])
def test_patch_dequant_add_requant_bit_exact(cuda, mode, inplace):
    gen = torch.Generator().manual_seed(3)
    n, d = 100, 256
    x = torch.randn(n, d, generator=gen)
    delta = (torch.randn(n, d, generator=gen) * 0.05)
    base = K.quantize(x.to(cuda), mode)
    c, s, z = OK.quantize(x.numpy(), mode)
    out = None if inplace else K.KiviTensor.empty(n, d, mode, cuda)
    res = K.patch(base, delta.to(cuda), out)
    c2, s2, z2 = OK.patch(c, s, z, delta.numpy(), mode)
    assert np.array_equal(_np(res.codes), c2)
    assert np.array_equal(_np(res.scale).view(np.uint16), s2.view(np.uint16))
    assert np.array_equal(_np(res.zero).view(np.uint16), z2.view(np.uint16))
    if not inplace:  # the base is untouched
        assert np.array_equal(_np(base.codes), c)


def test_patch_bf16_delta_and_error_bound(cuda):
    gen = torch.Generator().manual_seed(4)
    n, d = 64, 128
    x = torch.randn(n, d, generator=gen)
    delta = (torch.randn(n, d, generator=gen) * 0.1).to(torch.bfloat16)
    base = K.quantize(x.to(cuda), "v")
    res = K.patch(base, delta.to(cuda), K.KiviTensor.empty(n, d, "v", cuda))
    got = _np(K.dequantize(res))
    want = OK.dequantize(*OK.patch(*OK.quantize(x.numpy(), "v"), delta.float().numpy(), "v"), "v")
    assert np.array_equal(got, want)
    # requantised within half a step of the exact sum
    exact = OK.dequantize(*OK.quantize(x.numpy(), "v"), "v") + delta.float().numpy()
    step = (exact.reshape(n, -1, 32).max(-1) - exact.reshape(n, -1, 32).min(-1)) / 15
    assert (np.abs(got - exact).reshape(n, -1, 32) <= 0.5 * step[..., None] + 1e-3 * np.abs(exact).max()).all()
