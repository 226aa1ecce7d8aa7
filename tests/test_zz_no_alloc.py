"""The allocation-free subspace entry point agrees with the workspace entry point.

``dkv_subspace_correct_noalloc`` serves callers that cannot allocate device memory at
the moment they need a correction — a serving framework that owns every device buffer
through its own pool, a plugin that is handed only its inputs and outputs, a thread that
must not wait on the allocator.  It keeps its scratch in a fixed 16 MiB device array
inside the library.  This test calls it through the C ABI, twice in a row (the second
call finds the first call's leftovers in the shared array), and compares both results
with ``dkv_subspace_correct`` on the same inputs, within the subspace tests' fp32
tolerance.  It also checks that a problem too large for the fixed array is refused
before anything runs.  The file is named so pytest collects it last.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

import deltakv_b200 as dkv
from deltakv_b200 import _lib as L
from deltakv_b200 import ops

pytestmark = pytest.mark.gpu


def _args(reused, fresh, probes, basis, corr, sub, mu, n, d):
    return L.SubspaceArgs(
        reused=reused.data_ptr(), fresh=fresh.data_ptr(), kv_dtype=L.DKV_F32, n_tokens=n, d=d,
        reused_row_stride=d, fresh_row_stride=d, probe_index=probes.data_ptr(), n_probes=probes.numel(),
        basis=basis.data_ptr(), rank=basis.shape[1], token_weights=None,
        corrected=corr.data_ptr(), out_dtype=L.DKV_F32, out_row_stride=d,
        subspace_out=sub.data_ptr(), orth_mu_out=mu.data_ptr(), workspace=None, workspace_bytes=0,
    )


def test_noalloc_matches_workspace_entry_point(cuda):
    gen = torch.Generator().manual_seed(11)
    n, n_kv, hd, r = 900, 4, 64, 16
    d = n_kv * hd
    reused = torch.randn(n, n_kv, hd, generator=gen)
    basis = torch.randn(d, r, generator=gen)
    fresh = reused + (torch.randn(n, r, generator=gen) * 0.1 @ basis.T).view(n, n_kv, hd) + 0.02
    probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.long), torch.randperm(n, generator=gen)[:90]]))
    reused, fresh, basis = reused.to(cuda), fresh.to(cuda), basis.to(cuda)
    ref_corr, ref_sub, ref_mu = dkv.subspace_correct(reused, fresh, probes.to(cuda), basis=basis, rank=r)

    idx = probes.to(device=cuda, dtype=torch.int32)
    for call in range(2):
        corr = torch.full((n, d), float("nan"), device=cuda)
        sub = torch.full((d,), float("nan"), device=cuda)
        mu = torch.full((d,), float("nan"), device=cuda)
        args = _args(reused, fresh, idx, basis, corr, sub, mu, n, d)
        rc = L.lib().dkv_subspace_correct_noalloc(C.byref(args), ops.stream_ptr())
        assert rc == L.DKV_OK, L.lib().dkv_status_string(rc)
        torch.cuda.synchronize()
        for got, ref in ((corr.view(n, n_kv, hd), ref_corr), (sub, ref_sub), (mu, ref_mu)):
            err = float((got - ref).norm() / (ref.norm() + 1e-30))
            assert err < 1e-5, (call, err)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    n, d, r = 1 << 20, 1024, 64  # ~270 MB of scratch, far beyond the fixed 16 MiB
    x = torch.zeros(1, device=cuda)
    args = L.SubspaceArgs(
        reused=x.data_ptr(), fresh=x.data_ptr(), kv_dtype=L.DKV_F32, n_tokens=n, d=d, reused_row_stride=d,
        fresh_row_stride=d, probe_index=None, n_probes=0, basis=x.data_ptr(), rank=r, token_weights=None,
        corrected=x.data_ptr(), out_dtype=L.DKV_F32, out_row_stride=d, subspace_out=None, orth_mu_out=None,
        workspace=None, workspace_bytes=0,
    )
    assert L.lib().dkv_subspace_correct_noalloc(C.byref(args), ops.stream_ptr()) == L.DKV_ERR_WORKSPACE
