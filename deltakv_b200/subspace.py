"""Subspace route on the B200 kernels.

Drop-in for ``deltakv.patches.subspace.subspace_correct`` (src/deltakv/patches/subspace.py:45-106)
and ``svd_basis`` (37-42).  The per-token work (residual, least-squares codes onto col(B),
fitted field, CacheBlend-style weights, probe override) runs in ``libdkv_b200.so``; the K
path's basis — the top right singular vectors of the probe residual — is a library SVD
(torch.linalg.svd on the device) of the gathered [n_probes, d] residual.
"""

from __future__ import annotations

import ctypes as C

import torch
from torch import Tensor

from deltakv_b200 import _lib as L
from deltakv_b200 import ops

MAX_RANK = 64

_ws_cache: dict[tuple, Tensor] = {}


def workspace_bytes(n_tokens: int, d: int, rank: int) -> int:
    out = C.c_int64(0)
    L.check(L.lib().dkv_subspace_workspace_bytes(n_tokens, d, rank, C.byref(out)), "dkv_subspace_workspace_bytes")
    return int(out.value)


def _workspace(device: torch.device, nbytes: int) -> Tensor:
    key = (str(device),)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def probe_residual(reused2: Tensor, fresh2: Tensor, idx: Tensor) -> Tensor:
    """``fresh[P] - reused[P]`` as fp32 ``[n_probes, d]`` (rows ``[n, d]`` views)."""
    out = torch.empty(idx.numel(), reused2.shape[1], dtype=torch.float32, device=reused2.device)
    rc = L.lib().dkv_subspace_probe_residual(
        reused2.data_ptr(), fresh2.data_ptr(), ops.dkv_dtype(reused2.dtype), reused2.stride(0), fresh2.stride(0),
        reused2.shape[0], reused2.shape[1], idx.data_ptr(), idx.numel(), out.data_ptr(), ops.stream_ptr(),
    )
    L.check(rc, "dkv_subspace_probe_residual")
    return out


def svd_basis(residual: Tensor, rank: int) -> Tensor:
    """Leading-r right singular vectors of ``residual [n, d]`` as ``[d, r]``."""
    r = max(1, min(int(rank), residual.shape[0], residual.shape[1]))
    _, _, vh = torch.linalg.svd(residual.float(), full_matrices=False)
    return vh[:r].T.to(residual.dtype).contiguous()


def _rows(t: Tensor) -> Tensor:
    r = t.reshape(t.shape[0], -1)
    if r.stride(1) != 1:
        r = r.contiguous()
    return r


def subspace_correct(reused: Tensor, fresh: Tensor, probe_index: Tensor, *, basis: Tensor | None = None,
                     rank: int = 8, token_weights: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """Correct ``reused`` toward ``fresh`` in a rank-r subspace plus an orthogonal shift.

    Returns ``(corrected [seq, n_kv, hd], subspace_offset [d], orth_mu [d])`` like the reference.
    """
    ops._require_cuda(reused, fresh)
    seq, n_kv, hd = reused.shape
    dev = reused.device
    idx = probe_index.to(device=dev, dtype=torch.int64).reshape(-1)
    if idx.numel():
        lo, hi = int(idx.min()), int(idx.max())
        if lo < -seq or hi >= seq:
            bad = hi if hi >= seq else lo
            raise IndexError(f"index {bad} is out of bounds for dimension 0 with size {seq}")
        idx = torch.where(idx < 0, idx + seq, idx)  # torch indexing semantics
    idx = idx.to(torch.int32).contiguous()
    rf, ff = _rows(reused), _rows(fresh)
    if ff.dtype != rf.dtype:
        ff = ff.to(rf.dtype)
    d = rf.shape[1]
    if basis is None:
        r_eff = min(rank, max(1, int(idx.numel()) - 1), d)
        basis = svd_basis(probe_residual(rf, ff, idx), r_eff) if idx.numel() >= 2 else None
    structured = basis is not None and basis.numel() > 0 and idx.numel() >= 1
    if structured:
        if basis.shape[0] != d:
            raise ValueError(f"basis d={basis.shape[0]} != kv d={d}")
        if basis.shape[1] > MAX_RANK:
            raise NotImplementedError(f"subspace rank {basis.shape[1]} > {MAX_RANK} is not built")
        b32 = basis.to(device=dev, dtype=torch.float32).contiguous()
        r = b32.shape[1]
    else:
        b32, r = None, 0
    out_dtype = reused.dtype if reused.dtype in (torch.float32, torch.float16, torch.bfloat16) else torch.float32
    corr = torch.empty(seq, d, dtype=out_dtype, device=dev)
    sub = torch.zeros(d, dtype=torch.float32, device=dev)
    mu = torch.zeros(d, dtype=torch.float32, device=dev)
    tw = None
    if token_weights is not None:
        tw = token_weights.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    nbytes = workspace_bytes(seq, d, r)
    ws = _workspace(dev, nbytes)
    args = L.SubspaceArgs(
        reused=rf.data_ptr(), fresh=ff.data_ptr(), kv_dtype=ops.dkv_dtype(rf.dtype), n_tokens=seq, d=d,
        reused_row_stride=rf.stride(0), fresh_row_stride=ff.stride(0),
        probe_index=idx.data_ptr() if idx.numel() else None, n_probes=idx.numel(),
        basis=ops.ptr(b32), rank=r, token_weights=ops.ptr(tw),
        corrected=corr.data_ptr(), out_dtype=ops.dkv_dtype(out_dtype), out_row_stride=corr.stride(0),
        subspace_out=sub.data_ptr(), orth_mu_out=mu.data_ptr(), workspace=ws.data_ptr(), workspace_bytes=ws.numel(),
    )
    L.check(L.lib().dkv_subspace_correct(C.byref(args), ops.stream_ptr()), "dkv_subspace_correct")
    res_dtype = reused.dtype
    return corr.view(seq, n_kv, hd).to(res_dtype), sub.to(res_dtype), mu.to(res_dtype)
