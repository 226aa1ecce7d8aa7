"""Test infrastructure: the exact branch as torch CPU operations, for the timed CPU baseline.

Same steps as `oracle.exact` (which is what parity is checked against) in the operations the
reference itself uses on the CPU, so that the baseline runs at the reference's own speed:

* RMSNorm: ``x * rsqrt(mean(x^2) + eps) * w`` (src/deltakv/model.py:54-56);
* ``exact_kv_patch``: codes = s (x A^T), Δ = codes B^T, RoPE (rotate-half) on ΔK
  (src/deltakv/patches/exact.py:14-63, deltas/factors.py:58-65, rope.py:55-63);
* ``materialize`` keeps the dense ΔK / ΔV (patches/tensors.py:105-123);
* ``scatter_into_paged``: ``pages[bid, :span] = pages[bid, :span] + delta`` per block of the
  table (src/deltakv/paged.py:8-43), here as one indexed read-add-write over all full blocks
  (the table holds distinct blocks) and one for the ragged last block.

Plus the stored-activation dequantisation the reference does not have (its activations are
fp32): fp8-e4m3 or f16 codes times the per-row scale.  Checked against `oracle.exact` by
`tests/test_oracle_exact_torch.py`.
"""
from __future__ import annotations

import torch


def dequant_x(xb: torch.Tensor, kind: str, scale: torch.Tensor | None) -> torch.Tensor:
    """``[rows, d]`` fp8-e4m3 (uint8 bits) / f16 codes -> fp32 times the row scale"""
    x = xb.view(torch.float8_e4m3fn).float() if kind == "e4m3" else xb.float()
    return x if scale is None else x * scale[:, None]


def rmsnorm(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    y = x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    return y if w is None else y * w


def rope_full(cos_half: torch.Tensor, sin_half: torch.Tensor, seq: int):
    """``[seq, 1, hd]`` cos / sin rows (both halves equal) from the half-width tables"""
    c = torch.cat([cos_half[:seq], cos_half[:seq]], dim=-1)[:, None, :]
    s = torch.cat([sin_half[:seq], sin_half[:seq]], dim=-1)[:, None, :]
    return c.contiguous(), s.contiguous()


def exact_kv_delta(xn: torch.Tensor, fk, fv, n_kv: int, hd: int, rope=None):
    """``(dK, dV)`` ``[seq, n_kv, hd]`` fp32; ``fk`` / ``fv`` = (A, B, scale) tensors; ``rope`` =
    full-width (cos, sin) rows from `rope_full`, or None"""
    seq = xn.shape[0]

    def apply(f):
        A, B, s = f
        return ((xn @ A.T) * s) @ B.T

    dk = apply(fk).view(seq, n_kv, hd)
    if rope is not None:
        c, s = rope
        h = hd // 2
        dk = dk * c + torch.cat([-dk[..., h:], dk[..., :h]], dim=-1) * s
    dv = apply(fv).view(seq, n_kv, hd)
    return dk, dv


def scatter_into_paged(delta: torch.Tensor, pages: torch.Tensor, table: torch.Tensor, block_size: int) -> None:
    """In place on ``pages [num_blocks, block_size, n_kv, hd]`` (any float dtype):
    ``pages[bid, :span] = round(fp32(pages[bid, :span]) + delta[rows of the block])``"""
    seq = delta.shape[0]
    full, tail = divmod(seq, block_size)
    need = full + (1 if tail else 0)
    if table.numel() < need:
        raise ValueError("block_table shorter than prefix")
    if full:
        ids = table[:full]
        blk = delta[: full * block_size].view(full, block_size, *delta.shape[1:])
        pages[ids] = (pages[ids].float() + blk).to(pages.dtype)
    if tail:
        bid = int(table[full])
        pages[bid, :tail] = (pages[bid, :tail].float() + delta[full * block_size:]).to(pages.dtype)
