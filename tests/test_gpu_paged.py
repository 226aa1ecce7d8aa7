"""Paged scatter/gather on the GPU: bit-exact against the reference's golden vectors."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deltakv_b200 as dkv
from deltakv_b200 import ops
from oracle import exact as OX
from tests.conftest import golden
from tests.helpers import bf16_from_bits, bits_from_bf16

pytestmark = pytest.mark.gpu


def test_paged_roundtrip_golden(cuda):
    g = golden("paged")
    delta = torch.from_numpy(g["rt_delta"]).to(cuda)
    cache = torch.zeros(8, 8, 2, 8, device=cuda)
    dkv.scatter_into_paged(delta, cache, list(g["rt_table"]), 8)
    assert np.array_equal(cache.cpu().numpy(), g["rt_cache_out"])
    got = dkv.gather_from_paged(cache, list(g["rt_table"]), 20, 8)
    assert np.array_equal(got.cpu().numpy(), g["rt_gather"])


@pytest.mark.parametrize("name", ["l4", "l5a", "l5b"])
def test_paged_bf16_layouts_golden(cuda, name):
    g = golden("paged")
    c = bf16_from_bits(g[f"{name}_in"], cuda)
    delta = torch.from_numpy(g[f"{name}_delta"]).to(cuda)
    kv = int(g[f"{name}_kv"])
    dkv.scatter_into_paged(delta, c, list(g["l_table"]), int(g["l_bs"]), kv_dim=kv)
    assert np.array_equal(bits_from_bf16(c), g[f"{name}_out"])
    got = dkv.gather_from_paged(c, list(g["l_table"]), 13, int(g["l_bs"]), kv_dim=kv)
    assert np.array_equal(bits_from_bf16(got), g[f"{name}_gather"])


def test_errors_match_reference(cuda):
    with pytest.raises(ValueError, match="block_table shorter than prefix"):
        dkv.scatter_into_paged(torch.zeros(20, 1, 8, device=cuda), torch.zeros(4, 8, 1, 8, device=cuda), [0, 1], 8)
    with pytest.raises(ValueError, match="unsupported paged KV layout"):
        dkv.scatter_into_paged(torch.zeros(4, 1, 8, device=cuda), torch.zeros(3, 4, 8, 1, 8, device=cuda), [0], 8)
    with pytest.raises(ValueError, match="CUDA"):
        dkv.scatter_into_paged(torch.zeros(4, 1, 8), torch.zeros(1, 8, 1, 8), [0], 8)


@pytest.mark.parametrize("pdt,ddt", [(torch.bfloat16, torch.float32), (torch.float16, torch.bfloat16),
                                     (torch.float32, torch.float16), (torch.bfloat16, torch.bfloat16)])
def test_batched_scatter_matches_oracle(cuda, pdt, ddt):
    gen = torch.Generator().manual_seed(7)
    lens = [0, 5, 16, 33, 1, 100]
    bs, h, d = 16, 3, 32
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    need = [(n + bs - 1) // bs for n in lens]
    nb = sum(need) + 4
    perm = torch.randperm(nb, generator=gen).numpy().astype(np.int32)
    tables = np.zeros((len(lens), max(need)), np.int32)
    k = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[k:k + n]
        k += n
    pages = (torch.randn(nb, bs, h, d, generator=gen)).to(pdt)
    delta = (torch.randn(int(cu[-1]), h, d, generator=gen) * 0.05).to(ddt)
    ref = pages.clone().float().numpy() if pdt != torch.bfloat16 else bits_from_bf16(pages).copy()
    kind = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[pdt]
    if pdt == torch.float16:
        ref = pages.numpy().copy()
    for b, n in enumerate(lens):
        if n:
            OX.scatter_into_paged(delta[cu[b]:cu[b + 1]].float().numpy(), ref, list(tables[b, :need[b]]), bs, kind=kind)
    seqs = ops.SeqBatchTensors(cu_seqlens=torch.from_numpy(cu).to(cuda), block_tables=torch.from_numpy(tables).to(cuda),
                               max_seq_len=max(lens))
    pg = pages.to(cuda)
    dkv.scatter_into_paged_batched(delta.to(cuda), pg, seqs, check=True)
    got = bits_from_bf16(pg) if pdt == torch.bfloat16 else pg.cpu().numpy()
    assert np.array_equal(got, ref)


def test_device_range_errors_are_reported(cuda):
    seqs = ops.SeqBatchTensors(cu_seqlens=torch.tensor([0, 20], dtype=torch.int32, device=cuda),
                               block_tables=torch.tensor([[0, 9]], dtype=torch.int32, device=cuda), max_seq_len=20)
    pages = torch.zeros(4, 16, 1, 8, device=cuda)
    with pytest.raises(dkv.DkvError, match="block id outside"):
        dkv.scatter_into_paged_batched(torch.ones(20, 1, 8, device=cuda), pages, seqs, check=True)
    # rows with a valid block were still written, the bad block was skipped
    assert float(pages[0].sum()) == 16 * 8
    assert float(pages[1:].abs().sum()) == 0.0
