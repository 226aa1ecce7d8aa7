"""RoPE tables for the fused patch kernel.

The kernel reads ``cos/sin[position, i]`` for ``i < head_dim/2`` (the reference builds
``emb = cat(freqs, freqs)``, so the second half repeats the first; src/deltakv/rope.py:35-45).
Tables are built on the CPU with the same torch operations as the reference, so the angles
and their cos/sin are bit-identical to ``RotaryEmbedding.cos_cached/sin_cached``.
"""

from __future__ import annotations

import torch
from torch import Tensor


class RotaryEmbedding:
    """Llama rotate-half RoPE tables (src/deltakv/rope.py:28-63), without the module."""

    def __init__(self, head_dim: int, max_seq: int = 8192, base: float = 10000.0):
        if head_dim % 2 != 0:
            raise ValueError("RoPE head_dim must be even")
        inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        t = torch.arange(max_seq, dtype=torch.float32)
        freqs = torch.outer(t, inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1)
        self.head_dim = head_dim
        self.max_seq = max_seq
        self.base = base
        self.inv_freq = inv_freq
        self.cos_cached = emb.cos()
        self.sin_cached = emb.sin()


_table_cache: dict[tuple, tuple[Tensor, Tensor]] = {}


def half_tables(rope, device: torch.device) -> tuple[Tensor, Tensor]:
    """``(cos, sin)`` as contiguous fp32 ``[max_seq, head_dim/2]`` on ``device``.

    ``rope`` is a reference ``RotaryEmbedding`` module, one of this package, or a
    ``(cos, sin)`` pair that is already half-width.
    """
    if isinstance(rope, tuple):
        c, s = rope
        return c.to(device=device, dtype=torch.float32).contiguous(), s.to(device=device, dtype=torch.float32).contiguous()
    cos_full, sin_full = rope.cos_cached, rope.sin_cached
    key = (id(rope), cos_full.data_ptr(), str(device))
    hit = _table_cache.get(key)
    if hit is not None:
        return hit
    hd = cos_full.shape[-1]
    out = (
        cos_full[:, : hd // 2].to(device=device, dtype=torch.float32).contiguous(),
        sin_full[:, : hd // 2].to(device=device, dtype=torch.float32).contiguous(),
    )
    _table_cache[key] = out
    return out


def max_positions(rope) -> int:
    if isinstance(rope, tuple):
        return int(rope[0].shape[0])
    return int(getattr(rope, "max_seq", rope.cos_cached.shape[0]))
