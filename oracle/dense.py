"""Oracle of the dense-delta (RL step) route (numpy fp32; TEST INFRASTRUCTURE ONLY).

The reference has no dense operator.  A full-rank weight delta dW goes through its exact
route as ``LowRankFactors(A=dW, B=I, scale=1)`` (src/deltakv/deltas/factors.py:61-67 with
src/deltakv/patches/exact.py:14-63), so ``dK = RoPE(x_normed @ dW_K^T)`` and
``dV = x_normed @ dW_V^T``, scattered with ``scatter_into_paged`` (src/deltakv/paged.py:8-43).
This module feeds exactly those factors to :func:`oracle.exact.exact_patch_paged`.
"""

from __future__ import annotations

import numpy as np

from oracle.exact import exact_patch_paged

F32 = np.float32


def dense_factors(dw_k: np.ndarray | None, dw_v: np.ndarray | None, scale_k: float = 1.0, scale_v: float = 1.0):
    """``(fk, fv)`` as the reference builds them for a dense delta: ``(A=dW, B=I, scale)``."""
    ref = dw_k if dw_k is not None else dw_v
    eye = np.eye(ref.shape[0], dtype=F32)
    fk = None if dw_k is None else (np.asarray(dw_k, F32), eye, scale_k)
    fv = None if dw_v is None else (np.asarray(dw_v, F32), eye, scale_v)
    return fk, fv


def dense_patch_paged(*, x: np.ndarray, norm_w: np.ndarray | None, eps: float, dw_k, dw_v,
                      cu_seqlens: np.ndarray, block_tables: np.ndarray, k_pages: list, v_pages: list,
                      n_kv: int, hd: int, rope=None, kind: str = "bf16", accumulate: bool = True,
                      scale_k: float = 1.0, scale_v: float = 1.0) -> None:
    """In place on ``k_pages[l]`` / ``v_pages[l]``; ``x`` ``[L, rows, d]`` fp32 values (the
    stored bf16 activations), ``dw_k[l]`` / ``dw_v[l]`` ``[n_kv*hd, d]`` or None."""
    n_layers = x.shape[0]
    factors = [dense_factors(None if dw_k is None else dw_k[l], None if dw_v is None else dw_v[l], scale_k, scale_v)
               for l in range(n_layers)]
    exact_patch_paged(x=np.asarray(x, F32), x_dtype="f32", x_scale=None, norm_w=norm_w, eps=eps, factors=factors,
                      cu_seqlens=cu_seqlens, block_tables=block_tables, k_pages=k_pages, v_pages=v_pages,
                      n_kv=n_kv, hd=hd, rope=rope, kind=kind, accumulate=accumulate)
