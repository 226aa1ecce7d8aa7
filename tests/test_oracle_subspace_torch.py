"""The torch CPU forms of the subspace route and the int4 format (timed CPU baselines) against
the numpy oracle."""
import numpy as np
import pytest
import torch

from oracle import kivi as OK
from oracle import subspace as OS
from oracle import subspace_torch as OST


@pytest.mark.parametrize("mode", ["v", "k"])
def test_kivi_torch_bit_exact(mode):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((96, 128)) * rng.random((96, 1)) * 3).astype(np.float32)
    x[5, :32] = 0.25  # a constant group: range clamped to 1e-8
    codes, s, z = OK.quantize(x, mode)
    tc, ts, tz = OST.quantize(torch.from_numpy(x), mode)
    assert np.array_equal(tc.numpy(), codes)
    assert np.array_equal(ts.numpy().view(np.uint16), s.view(np.uint16))
    assert np.array_equal(tz.numpy().view(np.uint16), z.view(np.uint16))
    d_np = OK.dequantize(codes, s, z, mode)
    d_t = OST.dequantize(tc, ts, tz, mode)
    assert np.array_equal(d_t.numpy().view(np.uint32), d_np.view(np.uint32))


def test_subspace_torch_matches_oracle():
    rng = np.random.default_rng(4)
    n, d, r = 512, 256, 8
    reused = rng.standard_normal((n, d)).astype(np.float32)
    B = (rng.standard_normal((d, r)) / np.sqrt(d)).astype(np.float32)
    fresh = (reused + rng.standard_normal((n, r)).astype(np.float32) @ B.T
             + 0.05 * rng.standard_normal((n, d)).astype(np.float32)).astype(np.float32)
    probes = np.sort(rng.permutation(n)[:50])
    c_o, s_o, m_o = OS.subspace_correct(reused.reshape(n, 2, 128), fresh.reshape(n, 2, 128), probes, basis=B)
    c_t, s_t, m_t = OST.subspace_correct(torch.from_numpy(reused), torch.from_numpy(fresh),
                                         torch.from_numpy(probes), torch.from_numpy(B))
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))  # noqa: E731
    assert rel(c_t.numpy(), c_o.reshape(n, d)) < 1e-6
    assert rel(s_t.numpy(), s_o) < 1e-5
    assert rel(m_t.numpy(), m_o) < 1e-5
