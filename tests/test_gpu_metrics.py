"""Per-layer measured error and compare_kv on the GPU vs the reference's golden values and the
oracle (compare_kv within 1e-6 absolute: the reference computes its norms in fp32)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200 import metrics, ops
from deltakv_b200.types import KVCache
from oracle.metrics import measured_error as oracle_error
from tests.conftest import golden

pytestmark = pytest.mark.gpu


def test_measured_error_golden(cuda):
    g = golden("errors")
    t = lambda a: torch.from_numpy(a).to(cuda)
    est = metrics.measured_error(KVCache(k=t(g["pk"]), v=t(g["pv"])), KVCache(k=t(g["fk"]), v=t(g["fv"])))
    assert np.allclose(est.per_layer, g["per_layer"], rtol=1e-5, atol=1e-9)
    assert abs(est.relative_kv_l2 - float(g["rel"])) <= 1e-5 * float(g["rel"])


def test_compare_kv_golden(cuda):
    g = golden("compare")
    t = lambda a: torch.from_numpy(a).to(cuda)
    rep = metrics.compare_kv(KVCache(k=t(g["pk"]), v=t(g["pv"])), KVCache(k=t(g["fk"]), v=t(g["fv"])))
    got = np.array([[x.relative_l2_k, x.relative_l2_v, x.cosine_k, x.cosine_v] for x in rep.layers])
    np.testing.assert_allclose(got, g["per_layer"], rtol=0, atol=1e-6)
    assert abs(rep.max_relative_l2 - float(g["max_rel"])) <= 1e-6
    assert abs(rep.mean_relative_l2 - float(g["mean_rel"])) <= 1e-6
    assert abs(rep.min_cosine - float(g["min_cos"])) <= 1e-6
    assert set(rep.as_dict()) >= {"max_relative_l2", "mean_relative_l2", "min_cosine", "next_token_kl"}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_compare_kv_bf16_cache_matches_oracle(cuda, dtype):
    from oracle.metrics import compare_kv as oracle_compare

    gen = torch.Generator().manual_seed(21)
    fk, fv = torch.randn(4, 300, 8, 128, generator=gen), torch.randn(4, 300, 8, 128, generator=gen)
    pk = (fk + 0.02 * torch.randn(fk.shape, generator=gen)).to(dtype)
    pv = (fv + 0.03 * torch.randn(fv.shape, generator=gen)).to(dtype)
    rep = metrics.compare_kv(KVCache(k=pk.to(cuda), v=pv.to(cuda)), KVCache(k=fk.to(cuda), v=fv.to(cuda)))
    rows, mx, mean, mn = oracle_compare(pk.float().numpy(), pv.float().numpy(), fk.numpy(), fv.numpy())
    got = np.array([[x.relative_l2_k, x.relative_l2_v, x.cosine_k, x.cosine_v] for x in rep.layers])
    np.testing.assert_allclose(got, rows, rtol=1e-5, atol=1e-7)
    assert abs(rep.min_cosine - mn) <= 1e-7 and abs(rep.max_relative_l2 - mx) <= 1e-5 * mx


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_measured_error_paged_matches_oracle(cuda, dtype):
    gen = torch.Generator().manual_seed(3)
    L_, n_kv, hd, bs = 3, 2, 64, 16
    lens = [5, 40, 0, 33]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    rows = int(cu[-1])
    need = [(n + bs - 1) // bs for n in lens]
    nb = sum(need) + 2
    perm = torch.randperm(nb, generator=gen).numpy().astype(np.int32)
    tables = np.zeros((len(lens), max(need)), np.int32)
    k = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[k:k + n]
        k += n
    caches = [torch.randn(2, nb, bs, n_kv, hd, generator=gen).to(dtype) for _ in range(L_)]
    fresh_k = torch.randn(L_, rows, n_kv, hd, generator=gen).to(dtype)
    fresh_v = torch.randn(L_, rows, n_kv, hd, generator=gen).to(dtype)
    # dense patched view through the block tables (oracle input)
    pk = np.zeros((L_, rows, n_kv, hd), np.float32)
    pv = np.zeros_like(pk)
    for l in range(L_):
        for b, n in enumerate(lens):
            for i in range(n):
                pk[l, cu[b] + i] = caches[l][0, tables[b, i // bs], i % bs].float().numpy()
                pv[l, cu[b] + i] = caches[l][1, tables[b, i // bs], i % bs].float().numpy()
    _, want = oracle_error(pk, pv, fresh_k.float().numpy(), fresh_v.float().numpy())
    seqs = ops.SeqBatchTensors(cu_seqlens=torch.from_numpy(cu).to(cuda), block_tables=torch.from_numpy(tables).to(cuda),
                               max_seq_len=max(lens))
    dev_caches = [c.to(cuda) for c in caches]
    got = metrics.measured_error_paged([c[0] for c in dev_caches], [c[1] for c in dev_caches], fresh_k.to(cuda),
                                       fresh_v.to(cuda), seqs, check=True).cpu().numpy()
    assert np.allclose(got, want, rtol=1e-5)
