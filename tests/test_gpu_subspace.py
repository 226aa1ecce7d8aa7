"""subspace_correct on the GPU vs the reference's golden vectors and the oracle.

Tolerance: fp32 inputs within rel-L2 1e-5 of the reference (both fp32 throughout; the
r x r solve order differs); bf16 inputs within 1e-3 of the oracle rounded to bf16.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deltakv_b200 as dkv
from oracle.subspace import subspace_correct as oracle_subspace
from tests.conftest import golden
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["t1", "t2", "v", "k"])
def test_subspace_golden(cuda, case):
    g = golden("subspace")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    basis = None
    if case == "t1" or (case in ("v", "k") and int(g[f"{case}_use_basis"])):
        basis = t(g[f"{case}_basis"])
    corr, sub, orth = dkv.subspace_correct(t(g[f"{case}_reused"]), t(g[f"{case}_fresh"]), t(g[f"{case}_probes"]),
                                           basis=basis, rank=int(g[f"{case}_rank"]))
    ref = g[f"{case}_corr"]
    tol = 1e-5 if basis is not None else 1e-4  # the K path goes through a device SVD
    assert rel_l2(corr.cpu().numpy(), ref) < tol
    assert np.abs(orth.cpu().numpy() - g[f"{case}_orth"]).max() < 1e-4 * (1 + np.abs(g[f"{case}_orth"]).max())
    assert np.abs(sub.cpu().numpy() - g[f"{case}_sub"]).max() < 1e-4 * (1 + np.abs(g[f"{case}_sub"]).max())
    # probes take the fresh value exactly
    pr = g[f"{case}_probes"]
    assert np.array_equal(corr.cpu().numpy()[pr], g[f"{case}_fresh"][pr])


@pytest.mark.parametrize("n,n_kv,hd,r,dtype,weights,probe_kind", [
    (700, 8, 128, 16, torch.float32, False, "random"),
    (513, 4, 64, 8, torch.bfloat16, False, "random"),
    (1000, 8, 128, 64, torch.float32, True, "random"),
    (300, 2, 64, 48, torch.float16, False, "dups"),
    (257, 4, 32, 32, torch.float32, False, "none"),
    (129, 4, 32, 0, torch.float32, False, "random"),
])
def test_subspace_matches_oracle(cuda, n, n_kv, hd, r, dtype, weights, probe_kind):
    gen = torch.Generator().manual_seed(n + r)
    d = n_kv * hd
    reused = torch.randn(n, n_kv, hd, generator=gen)
    B = torch.randn(d, max(r, 1), generator=gen)
    codes = torch.randn(n, max(r, 1), generator=gen) * 0.1
    fresh = reused + (codes @ B.T).view(n, n_kv, hd) + 0.05 * torch.randn(d, generator=gen).view(1, n_kv, hd) \
        + 0.01 * torch.randn(n, n_kv, hd, generator=gen)
    reused, fresh = reused.to(dtype), fresh.to(dtype)
    if probe_kind == "random":
        probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.long), torch.randperm(n, generator=gen)[: n // 10]]))
    elif probe_kind == "dups":
        probes = torch.tensor([0, 5, 5, 9, 17, 17, 17, 40])
    else:
        probes = torch.zeros(0, dtype=torch.long)
    tw = torch.rand(n, generator=gen) if weights else None
    basis = B if r > 0 else None
    ref = oracle_subspace(reused.float().numpy(), fresh.float().numpy(), probes.numpy(),
                          basis=None if basis is None else basis.numpy(), rank=max(r, 1),
                          token_weights=None if tw is None else tw.numpy())
    out = dkv.subspace_correct(reused.to(cuda), fresh.to(cuda), probes.to(cuda),
                               basis=None if basis is None else basis.to(cuda), rank=max(r, 1),
                               token_weights=None if tw is None else tw.to(cuda))
    corr = out[0].float().cpu().numpy()
    ref_corr = torch.from_numpy(ref[0]).to(dtype).float().numpy()
    tol = 1e-5 if dtype == torch.float32 else 2e-3
    if r == 0:
        tol = max(tol, 1e-4)  # device SVD basis vs numpy's
    assert rel_l2(corr, ref_corr) < tol
    if probes.numel():
        assert np.array_equal(out[0].cpu()[probes].float().numpy(), fresh[probes].float().numpy())


def test_subspace_errors(cuda):
    x = torch.randn(10, 2, 8, device=cuda)
    with pytest.raises(ValueError, match="basis d=5 != kv d=16"):
        dkv.subspace_correct(x, x + 1, torch.tensor([0, 1], device=cuda), basis=torch.randn(5, 2, device=cuda))
    with pytest.raises(IndexError):
        dkv.subspace_correct(x, x + 1, torch.tensor([0, 10], device=cuda), basis=torch.randn(16, 2, device=cuda))


def test_subspace_batched_matches_single_calls(cuda):
    """One batched call over problems of mixed rank, dtype and weights gives the single calls'
    results; a batch the batched form does not take (d = 16) runs one problem at a time."""
    gen = torch.Generator().manual_seed(31)
    probs, d = [], 256
    for j, (r, dt, weights) in enumerate([(8, torch.bfloat16, False), (64, torch.float32, True),
                                          (0, torch.float16, False), (16, torch.bfloat16, False)]):
        n = 300 + 97 * j
        reused = torch.randn(n, 4, 64, generator=gen).to(dt)
        fresh = (reused.float() + 0.1 * torch.randn(n, 4, 64, generator=gen)).to(dt)
        probes = torch.unique(torch.randperm(n, generator=gen)[: n // 8])
        probs.append(dict(reused=reused.to(cuda), fresh=fresh.to(cuda), probe_index=probes.to(cuda),
                          basis=(torch.randn(d, r, generator=gen) / 16).to(cuda) if r else None, rank=max(r, 4),
                          token_weights=torch.rand(n, generator=gen).to(cuda) if weights else None))
    for group in (probs[:2], [probs[0], probs[3]]):  # same dtype per batched launch; mixed falls back
        got = dkv.subspace_correct_batched(group)
        for p, (corr, sub, mu) in zip(group, got):
            ref = dkv.subspace_correct(p["reused"], p["fresh"], p["probe_index"], basis=p["basis"],
                                       rank=p["rank"], token_weights=p["token_weights"])
            # the probe sums are atomics over a grid sized by the batch: equal up to summation
            # order (fp32 ~1e-7, which can move a 16-bit output across a rounding boundary)
            tol = 1e-5 if p["reused"].dtype == torch.float32 else 1e-4
            for a, b in zip((corr, sub, mu), ref):
                a, b = a.float().cpu().numpy(), b.float().cpu().numpy()
                assert rel_l2(a, b) < tol, rel_l2(a, b)
    small = [dict(reused=torch.randn(40, 2, 8, device=cuda), fresh=torch.randn(40, 2, 8, device=cuda),
                  probe_index=torch.tensor([1, 5, 9], device=cuda), rank=2)]
    got = dkv.subspace_correct_batched(small)
    ref = dkv.subspace_correct(small[0]["reused"], small[0]["fresh"], small[0]["probe_index"], rank=2)
    assert torch.allclose(got[0][0], ref[0], atol=1e-5)
