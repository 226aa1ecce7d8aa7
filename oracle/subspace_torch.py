"""Test infrastructure: the subspace route and the int4 KIVI format as torch CPU operations, for
the timed CPU baselines.

Same steps as `oracle.subspace` and `oracle.kivi` (which parity is checked against), in the
torch operations the reference itself uses, so that the baselines run at the reference's own
CPU speed:

* ``subspace_correct``: the reference's `subspace_correct` with a given basis
  (src/deltakv/patches/subspace.py:45-106, `_solve_codes` 21-34): rhs = R B,
  codes = solve(BᵀB + 1e-6 I, rhsᵀ)ᵀ, fitted = codes Bᵀ, orth_mu over the probes, the CacheBlend
  weight w = min(‖R‖ / mean ‖R‖, 1), probes take the fresh rows;
* ``quantize`` / ``dequantize``: the int4 format of `oracle.kivi` (per-group min / max as in the
  reference's `metrics._minmax_quantize`, src/deltakv/metrics.py:115-132, with fp16 scale and
  zero rounded before the codes are formed; V groups 32 channels of a token, K groups 32 tokens
  of a channel), each step one IEEE fp32 operation as in the numpy form.

Checked against the numpy forms by `tests/test_oracle_subspace_torch.py`.
"""
from __future__ import annotations

import torch

G = 32


def subspace_correct(reused: torch.Tensor, fresh: torch.Tensor, idx: torch.Tensor, basis: torch.Tensor):
    """``reused``, ``fresh`` ``[n, d]`` fp32, ``idx`` int64 probe rows, ``basis`` ``[d, r]`` ->
    ``(corrected [n, d], subspace [d], orth_mu [d])``"""
    residual = fresh - reused
    rp = residual[idx]
    gram = basis.T @ basis
    eye = torch.eye(gram.shape[0], dtype=gram.dtype)
    codes = torch.linalg.solve(gram + 1e-6 * eye, (residual @ basis).T).T
    fitted = codes @ basis.T
    subspace = codes.mean(dim=0) @ basis.T
    orth_mu = (rp - fitted[idx]).mean(dim=0)
    dist = residual.norm(dim=-1)
    w = (dist / dist.mean().clamp_min(1e-8)).clamp(max=1.0)
    corr = reused + fitted + w.unsqueeze(-1) * orth_mu.unsqueeze(0)
    corr[idx] = fresh[idx]
    return corr, subspace, orth_mu


def _groups(x: torch.Tensor, mode: str) -> torch.Tensor:
    """``[n, d]`` -> ``[groups..., 32]`` views of the quantisation groups (K: n a multiple of 32)"""
    n, d = x.shape
    if mode == "v":
        return x.view(n, d // G, G)
    return x.view(n // G, G, d).transpose(1, 2)


def quantize(x: torch.Tensor, mode: str):
    """``x [n, d]`` fp32 -> ``(codes [n, d/2] uint8, scale fp16, zero fp16)``; V scale / zero
    ``[n, d/32]``, K ``[n/32, d]`` (K: n a multiple of 32)"""
    g = _groups(x, mode)
    lo = g.amin(dim=-1)
    hi = g.amax(dim=-1)
    s16 = (torch.clamp_min(hi - lo, 1e-8) / 15.0).to(torch.float16)
    z16 = lo.to(torch.float16)
    s = s16.float().unsqueeze(-1)
    z = z16.float().unsqueeze(-1)
    q = torch.round((g - z) / s).clamp(0, 15)
    q = torch.where(s > 0, q, torch.zeros_like(q)).to(torch.uint8)
    q = q.reshape(x.shape) if mode == "v" else q.transpose(1, 2).reshape(x.shape)
    codes = q[:, 0::2] | (q[:, 1::2] << 4)
    return codes, s16, z16


def dequantize(codes: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, mode: str) -> torch.Tensor:
    n, h = codes.shape
    q = torch.empty(n, 2 * h, dtype=torch.float32)
    q[:, 0::2] = (codes & 0xF).float()
    q[:, 1::2] = (codes >> 4).float()
    g = _groups(q, mode)
    out = g * scale.float().unsqueeze(-1) + zero.float().unsqueeze(-1)
    return out.reshape(n, 2 * h) if mode == "v" else out.transpose(1, 2).reshape(n, 2 * h)
