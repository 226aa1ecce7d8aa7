"""Dense-delta (RL step) route: full-rank dW on k_proj / v_proj as one tensor-core GEMM.

The reference has no separate dense operator; a dense delta goes through the exact route as
``LowRankFactors(A=dW, B=I, scale=1)`` (src/deltakv/patches/exact.py:14-63,
src/deltakv/factors.py:61-67), i.e. ``dK = RoPE(x_normed @ dW_K^T)``, ``dV = x_normed @ dW_V^T``,
followed by ``scatter_into_paged`` (src/deltakv/paged.py:8-43).  :class:`DensePatcher` does
all of it for every layer and sequence in one launch of ``dkv_dense_patch_paged``.
"""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor

from deltakv_b200 import ops
from deltakv_b200.rope import half_tables


class DensePatcher:
    """``pack`` once per delta (bf16 operand, RMSNorm weight folded in); ``apply`` per batch."""

    def __init__(self, d_model: int, n_kv_heads: int, head_dim: int, *, rope=None, norm_eps: float = 1e-6):
        self.d_model, self.n_kv, self.hd = d_model, n_kv_heads, head_dim
        self.rope = rope
        self.norm_eps = norm_eps
        self.geom = ops.dense_geometry(d_model, n_kv_heads, head_dim)

    def pack(self, dw_k: Tensor | None, dw_v: Tensor | None, *, scale_k: float = 1.0, scale_v: float = 1.0,
             norm_weight: Tensor | None = None, out: Tensor | None = None) -> Tensor:
        return ops.pack_dense_delta(self.geom, dw_k, dw_v, scale_k=scale_k, scale_v=scale_v,
                                    norm_weight=norm_weight, out=out)

    def norm_scale(self, x: Tensor) -> Tensor:
        """Per-row RMSNorm factor of pre-norm activations (compute once when X is captured)."""
        return ops.row_inv_rms(x, self.norm_eps)

    def apply(self, x: Tensor, packed: Tensor, k_pages: Sequence[Tensor], v_pages: Sequence[Tensor],
              seqs: ops.SeqBatchTensors, *, x_scale: Tensor | None = None, do_k: bool = True,
              do_v: bool = True, accumulate: bool = True, check: bool = False) -> None:
        cos = sin = None
        if self.rope is not None:
            cos, sin = half_tables(self.rope, x.device)
        st = ops.status_word(x.device)
        ops.dense_patch_paged(self.geom, x, packed, k_pages, v_pages, seqs, x_scale=x_scale,
                              rope_cos=cos, rope_sin=sin, do_k=do_k, do_v=do_v,
                              accumulate=accumulate, status=st)
        if check:
            st.raise_if_set("DensePatcher.apply")
