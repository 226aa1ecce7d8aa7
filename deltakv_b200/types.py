"""Data containers with the reference's field names, so objects from either side work.

The operators in this package duck-type their arguments: a reference ``LowRankFactors``
(``.A``, ``.B``, ``.scale``), ``LayerDelta`` (``.get(name)``), ``KVCache`` (``.k``, ``.v``,
``.version``) or ``LowRankKVPatch`` is accepted as well as the classes below, which
mirror src/deltakv/deltas/factors.py:11-75, src/deltakv/deltas/descriptor.py:23-45 and
src/deltakv/patches/tensors.py:13-55,105-123.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
from torch import Tensor


@dataclass
class LowRankFactors:
    """PEFT LoRA factors: ``A [rank, in]``, ``B [out, rank]``, dW = scale * B @ A."""

    A: Tensor
    B: Tensor
    scale: float = 1.0
    name: str = ""

    def __post_init__(self) -> None:
        if self.A.ndim != 2 or self.B.ndim != 2:
            raise ValueError("A and B must be rank-2")
        if self.A.shape[0] != self.B.shape[1]:
            raise ValueError(f"rank mismatch: A {tuple(self.A.shape)} vs B {tuple(self.B.shape)}")

    @property
    def rank(self) -> int:
        return int(self.A.shape[0])

    @property
    def in_features(self) -> int:
        return int(self.A.shape[1])

    @property
    def out_features(self) -> int:
        return int(self.B.shape[0])


@dataclass
class LayerDelta:
    layer_idx: int
    projections: dict[str, Any] = field(default_factory=dict)

    def get(self, name: str):
        return self.projections.get(name)


@dataclass
class KVCache:
    """Dense KV of one prefix, ``[n_layers, seq, n_kv_heads, head_dim]``."""

    k: Tensor
    v: Tensor
    version: Any = None
    token_ids: Tensor | None = None

    def __post_init__(self) -> None:
        if self.k.shape != self.v.shape:
            raise ValueError(f"K/V shape mismatch {tuple(self.k.shape)} vs {tuple(self.v.shape)}")

    @property
    def n_layers(self) -> int:
        return int(self.k.shape[0])

    @property
    def seq_len(self) -> int:
        return int(self.k.shape[1])

    @property
    def n_kv_heads(self) -> int:
        return int(self.k.shape[2])

    @property
    def head_dim(self) -> int:
        return int(self.k.shape[3])

    def layer(self, idx: int) -> tuple[Tensor, Tensor]:
        return self.k[idx], self.v[idx]

    def clone(self) -> "KVCache":
        return KVCache(k=self.k.clone(), v=self.v.clone(), version=self.version,
                       token_ids=None if self.token_ids is None else self.token_ids.clone())


@dataclass
class LowRankKVPatch:
    """dK / dV of one layer: dense (post-RoPE) tensors or codes @ basis.T."""

    layer_idx: int
    k_codes: Tensor | None
    k_basis: Tensor | None
    v_codes: Tensor | None
    v_basis: Tensor | None
    k_dense: Tensor | None = None
    v_dense: Tensor | None = None

    def materialize(self, n_kv_heads: int, head_dim: int) -> tuple[Tensor, Tensor]:
        from deltakv_b200.exact import materialize_codes

        def one(dense, codes, basis):
            if dense is not None:
                return dense
            if codes is None or basis is None:
                raise ValueError("patch is empty")
            return materialize_codes(codes, basis, n_kv_heads, head_dim)

        return one(self.k_dense, self.k_codes, self.k_basis), one(self.v_dense, self.v_codes, self.v_basis)

    def nbytes(self) -> int:
        n = 0
        for t in (self.k_codes, self.k_basis, self.v_codes, self.v_basis, self.k_dense, self.v_dense):
            if t is not None:
                n += t.numel() * t.element_size()
        return n


def as_factors(f) -> tuple[Tensor, Tensor, float] | None:
    """``(A, B, scale)`` of any LoRA-factor-like object, or None."""
    if f is None:
        return None
    return f.A, f.B, float(getattr(f, "scale", 1.0))


def kv_factors(layer) -> tuple:
    """``(k, v)`` factor triples of a LayerDelta-like object (``get("k_proj")``)."""
    if layer is None:
        return None, None
    return as_factors(layer.get("k_proj")), as_factors(layer.get("v_proj"))
