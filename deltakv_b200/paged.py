"""Drop-ins for ``deltakv.paged`` (src/deltakv/paged.py:8-70) on the B200 kernels.

Same signatures, layouts, in-place additive semantics and error messages as the
reference; the per-block Python loop becomes one kernel launch.  Results are
bit-identical: each element is ``round(fp32(page) + fp32(delta))`` in the page dtype.
"""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor

from deltakv_b200 import ops


def _normalise_table(block_table: Sequence[int], num_blocks: int) -> list[int]:
    # torch indexing accepts negative block ids (pages[-1] is the last block)
    out = []
    for bid in block_table:
        b = int(bid)
        if b < -num_blocks or b >= num_blocks:
            raise IndexError(f"index {b} is out of bounds for dimension 0 with size {num_blocks}")
        out.append(b % num_blocks)
    return out


def scatter_into_paged(delta: Tensor, cache: Tensor, block_table: list[int], block_size: int, *,
                       kv_dim: int = 0) -> None:
    """Add ``delta [seq, n_kv_heads, head_dim]`` into a paged cache, in place.

    Layouts: ``[num_blocks, block_size, h, d]``, ``[2, num_blocks, block_size, h, d]``
    (``kv_dim`` picks K=0 / V=1) and ``[num_blocks, 2, block_size, h, d]``.
    """
    seq = delta.shape[0]
    n_blocks_needed = (seq + block_size - 1) // block_size
    if len(block_table) < n_blocks_needed:
        raise ValueError("block_table shorter than prefix")
    pages = ops.page_view(cache, kv_dim)
    if seq == 0:
        return
    if block_size > pages.shape[1]:
        raise ValueError(f"block_size {block_size} exceeds the cache's {pages.shape[1]} slots per block")
    table = _normalise_table(list(block_table)[:n_blocks_needed], pages.shape[0])
    seqs = ops.SeqBatchTensors.single(seq, table, pages.device)
    # the kernel reads slot i % block_size of block i // block_size, as the reference does
    view = pages if block_size == pages.shape[1] else pages[:, :block_size]
    ops.scatter_paged(delta, view, seqs)


def gather_from_paged(cache: Tensor, block_table: list[int], seq_len: int, block_size: int, *,
                      kv_dim: int = 0) -> Tensor:
    """Inverse of :func:`scatter_into_paged`: ``[seq_len, n_kv_heads, head_dim]``.

    Rows past the end of a short block table stay zero, as in the reference.
    """
    pages = ops.page_view(cache, kv_dim)
    n_kv, hd = pages.shape[-2], pages.shape[-1]
    out = pages.new_zeros(seq_len, n_kv, hd)
    n_blocks_needed = (seq_len + block_size - 1) // block_size
    table = _normalise_table(list(block_table)[:n_blocks_needed], pages.shape[0])
    covered = min(seq_len, len(table) * block_size)
    if covered == 0:
        return out
    view = pages if block_size == pages.shape[1] else pages[:, :block_size]
    seqs = ops.SeqBatchTensors.single(covered, table, pages.device)
    ops.gather_paged(view, seqs, out)
    return out


def scatter_into_paged_batched(delta: Tensor, pages: Tensor, seqs: ops.SeqBatchTensors,
                               check: bool = False) -> None:
    """Many sequences in one launch: ``delta`` rows follow ``seqs.cu_seqlens``.

    With ``check=True`` device-side range errors (short table, block id out of range) are
    raised after a synchronisation; otherwise they are recorded in the status word only.
    """
    st = ops.status_word(pages.device)
    ops.scatter_paged(delta, pages, seqs, st)
    if check:
        st.raise_if_set("scatter_into_paged_batched")
