"""The C ABI library loads here (no GPU) and exports every symbol the header declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def _declared() -> set[str]:
    text = (ROOT / "include" / "dkv_b200.h").read_text()
    return set(re.findall(r"^\s*(?:const\s+)?(?:int|void|char\s*\*|const char\s*\*)\s*\*?\s*(dkv_\w+)\s*\(", text, re.M))


def test_header_declares_the_bound_symbols():
    from deltakv_b200 import _lib

    assert _declared() == set(_lib.EXPORTED)


def test_library_loads_and_exports_all_symbols():
    from deltakv_b200 import _lib

    lib = _lib.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.dkv_abi_version() == _lib.ABI_VERSION == 2
    assert lib.dkv_status_string(-2).decode() == "block_table shorter than prefix"
    assert lib.dkv_status_string(-3).decode() == "unsupported paged KV layout"


def test_struct_layouts_match_the_header():
    from deltakv_b200 import _lib as L

    # sizes of the ABI structs under the x86-64 SysV layout of the C header
    assert ctypes.sizeof(L.PagedCache) == 56
    assert ctypes.sizeof(L.SeqBatch) == 48
    assert ctypes.sizeof(L.ExactGeometry) == 24


def test_packed_bytes_host_query():
    from deltakv_b200 import ops

    g = ops.exact_geometry(4096, 8, 128, torch.float8_e4m3fn, 16, 16)
    n = ops.packed_bytes(g)
    # header 256 + A (32 stages x (3 e4m3 terms x 2 projections x 16 rows) x 128 B)
    # + 2 x B (16 passes x 1 k-step x 2 KiB)
    assert n == 256 + 32 * 96 * 128 + 2 * 16 * 2048
    # ranks above 32 use the mma.sync image: f16 rows of 128 k per stage
    g64 = ops.exact_geometry(4096, 8, 128, torch.float8_e4m3fn, 64, 64)
    assert ops.packed_bytes(g64) == 256 + 32 * 128 * 256 + 2 * 16 * 4 * 2048
    with pytest.raises(Exception, match="unsupported"):
        ops.packed_bytes(ops.exact_geometry(4096, 8, 96, torch.float8_e4m3fn, 16, 16))


def test_calls_without_a_gpu_fail_cleanly_on_bad_arguments():
    from deltakv_b200 import _lib as L

    lib = L.lib()
    assert lib.dkv_scatter_paged(None, 0, 0, 0, None, None, None, None) == L.DKV_ERR_INVALID_ARGUMENT
    assert lib.dkv_exact_patch_paged(None, None) == L.DKV_ERR_INVALID_ARGUMENT
    # the split-precision thin GEMM checks its shape and layout before touching memory
    sg = lambda a, lda, tr, b, ldb, c, ldc, m, n, k: lib.dkv_split_gemm_batched(a, 0, lda, tr, b, 0, ldb, c, 0, ldc,
                                                                               1, m, n, k, None)
    p16 = 1 << 20  # a 16-byte-aligned stand-in address, never dereferenced on these paths
    assert sg(p16, 64, 0, p16, 24, p16, 24, 8, 24, 64) == L.DKV_ERR_UNSUPPORTED    # n not a multiple of 16
    assert sg(p16, 64, 0, p16, 112, p16, 112, 8, 112, 64) == L.DKV_ERR_UNSUPPORTED  # n above 96
    assert sg(p16 + 4, 64, 0, p16, 16, p16, 16, 8, 16, 64) == L.DKV_ERR_ALIGNMENT  # a not 16-byte aligned
    assert sg(p16, 66, 0, p16, 16, p16, 16, 8, 16, 64) == L.DKV_ERR_ALIGNMENT      # lda not whole float4s
    assert sg(p16, 64, 0, p16, 16, p16, 16, 8, 16, 62) == L.DKV_ERR_ALIGNMENT      # k % 4
    assert sg(p16, 64, 1, p16, 16, p16, 16, 6, 16, 64) == L.DKV_ERR_ALIGNMENT      # m % 4 with trans_a
    assert sg(None, 64, 0, p16, 16, p16, 16, 8, 16, 64) == L.DKV_ERR_INVALID_ARGUMENT
    assert sg(p16, 64, 0, p16, 16, p16, 16, 0, 16, 64) == L.DKV_OK                 # nothing to do


def test_page_view_matches_reference_layout_dispatch():
    from deltakv_b200.ops import page_view

    c4 = torch.zeros(3, 4, 2, 8)
    assert page_view(c4).shape == (3, 4, 2, 8)
    c5a = torch.zeros(2, 3, 4, 2, 8)
    assert page_view(c5a, 1).data_ptr() == c5a[1].data_ptr()
    c5b = torch.zeros(3, 2, 4, 2, 8)
    assert page_view(c5b, 1).stride() == c5b[:, 1].stride()
    with pytest.raises(ValueError, match="unsupported paged KV layout"):
        page_view(torch.zeros(3, 3, 4, 2, 8))


def test_cpu_tensors_are_rejected():
    import deltakv_b200 as dkv

    with pytest.raises(ValueError, match="CUDA"):
        dkv.scatter_into_paged(torch.zeros(4, 1, 8), torch.zeros(1, 8, 1, 8), [0], 8)


def test_block_table_rows_get_standard_strides():
    """Without per-row lengths the ABI reads a row's length from its stride: one-row tables
    from numpy's x[None] (row stride 0) and column slices are given standard strides."""
    import numpy as np
    import torch

    from deltakv_b200.ops import SeqBatchTensors

    cu = torch.tensor([0, 80], dtype=torch.int32)
    one = torch.from_numpy(np.arange(5, dtype=np.int32)[None])
    s = SeqBatchTensors(cu_seqlens=cu, block_tables=one, max_seq_len=80)
    assert s.block_tables.stride(0) == 5 and torch.equal(s.block_tables, one)
    wide = torch.arange(30, dtype=torch.int32).view(3, 10)[:, :4]
    s = SeqBatchTensors(cu_seqlens=torch.tensor([0, 1, 2, 3], dtype=torch.int32), block_tables=wide, max_seq_len=1)
    assert s.block_tables.stride(0) == 4 and torch.equal(s.block_tables, wide)
    lens = torch.tensor([4, 4, 4], dtype=torch.int32)
    s = SeqBatchTensors(cu_seqlens=torch.tensor([0, 1, 2, 3], dtype=torch.int32), block_tables=wide, max_seq_len=1,
                        table_lens=lens)
    assert s.block_tables.stride(0) == 10  # explicit lengths: the caller's strides are kept
