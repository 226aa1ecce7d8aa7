"""Exact / zeroth-order patch route on the fused B200 kernel.

Drop-ins with the reference's signatures:

* :func:`exact_kv_patch`        src/deltakv/patches/exact.py:14-63
* :func:`zeroth_order_patches`  src/deltakv/patches/exact.py:66-94
* :func:`apply_layer_patches`   src/deltakv/patches/compose.py:29-34

and the batched paged entry point the engine and the connector use,
:class:`ExactPatcher` — one launch for every (layer, sequence) of a cache, straight from
stored activations into the paged K/V blocks (the fused form of the engine's exact branch,
src/deltakv/engine.py:263-288, followed by DeltaKVConnector.patch_paged's scatter).

The drop-ins return dense ``k_dense`` / ``v_dense`` (the reference keeps V as codes and
basis); ``materialize`` gives the same ``(dK, dV)``.
"""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor

from deltakv_b200 import _lib as L
from deltakv_b200 import ops
from deltakv_b200.rope import half_tables, max_positions
from deltakv_b200.types import KVCache, LowRankKVPatch, as_factors, kv_factors

MAX_RANK_PER_LAUNCH = 64


class ExactPatcher:
    """Fused exact-route patcher for one model geometry.

    ``pack`` turns per-layer LoRA factors into the kernel's operand image (do it once per
    committed delta); ``apply`` patches ``L`` layers of a batch of sequences in one launch.
    """

    def __init__(self, d_model: int, n_kv_heads: int, head_dim: int, *, rank_k: int, rank_v: int,
                 x_dtype: torch.dtype = torch.float8_e4m3fn, rope=None, norm_eps: float = 1e-6):
        if rank_k > MAX_RANK_PER_LAUNCH or rank_v > MAX_RANK_PER_LAUNCH:
            raise ValueError(f"ranks above {MAX_RANK_PER_LAUNCH} need several launches (use exact_kv_patch)")
        self.d_model, self.n_kv, self.hd = d_model, n_kv_heads, head_dim
        self.rank_k, self.rank_v = rank_k, rank_v
        self.x_dtype = x_dtype
        self.rope = rope
        self.norm_eps = norm_eps
        self.geom = ops.exact_geometry(d_model, n_kv_heads, head_dim, x_dtype, rank_k, rank_v)
        self.packed_bytes = ops.packed_bytes(self.geom)

    def pack(self, a_k: Tensor | None, b_k: Tensor | None, a_v: Tensor | None, b_v: Tensor | None,
             scale_k: float = 1.0, scale_v: float = 1.0, norm_weight: Tensor | None = None,
             out: Tensor | None = None) -> Tensor:
        return ops.pack_factors(self.geom, a_k, b_k, a_v, b_v, scale_k, scale_v, norm_weight, out)

    def apply(self, x: Tensor, packed: Tensor, k_pages: Sequence[Tensor], v_pages: Sequence[Tensor],
              seqs: ops.SeqBatchTensors, *, x_scale: Tensor | None = None, apply_norm: bool = False,
              accumulate: bool = True, check: bool = False, x_sumsq: Tensor | None = None) -> None:
        """``x_sumsq``: the per-row sums of squared codes :func:`deltakv_b200.ops.quantize_rows`
        writes with ``with_sumsq=True``; with ``apply_norm`` the RMSNorm then uses them rather
        than forming them on the tensor cores (less tensor work, a higher clock under the
        power cap)."""
        dev = x.device
        cos = sin = None
        if self.rope is not None:
            cos, sin = half_tables(self.rope, dev)
        st = ops.status_word(dev)
        ops.exact_patch_paged(self.geom, x, packed, k_pages, v_pages, seqs, x_scale=x_scale,
                              apply_norm=apply_norm, norm_eps=self.norm_eps, rope_cos=cos, rope_sin=sin,
                              accumulate=accumulate, status=st, x_sumsq=x_sumsq)
        if check:
            st.raise_if_set("ExactPatcher.apply")


def _dense_pages(t: Tensor) -> Tensor:
    """A dense ``[seq, n_kv, hd]`` tensor viewed as one block of ``seq`` slots."""
    return t.unsqueeze(0)


def _rank_chunks(f):
    if f is None:
        return [None]
    A, B, s = f
    r = A.shape[0]
    if r <= MAX_RANK_PER_LAUNCH:
        return [f]
    return [(A[i:i + MAX_RANK_PER_LAUNCH], B[:, i:i + MAX_RANK_PER_LAUNCH], s) for i in range(0, r, MAX_RANK_PER_LAUNCH)]


def _dense_delta(x_list: list[Tensor], factors: list[tuple], n_kv: int, hd: int, rope, positions,
                 out_k: list[Tensor], out_v: list[Tensor], accumulate_first: bool) -> None:
    """dK/dV of several layers (same seq, same ranks) into dense fp32 outputs, one launch per
    rank chunk.  ``factors[l] = (fk, fv)`` as (A, B, scale) triples or None."""
    dev = x_list[0].device
    seq, d = x_list[0].shape
    x = torch.stack(x_list) if len(x_list) > 1 else x_list[0].unsqueeze(0)
    xq, xs = ops.quantize_rows(x, torch.float16)
    cos = sin = None
    if rope is not None:
        n_pos = seq if positions is None else int(positions.max().item()) + 1
        if n_pos > max_positions(rope):
            raise ValueError(f"seq_len {n_pos} exceeds RoPE cache {max_positions(rope)}")
        cos, sin = half_tables(rope, dev)
    pos = None
    if positions is not None:
        pos = positions.to(device=dev, dtype=torch.int32).contiguous()
    seqs = ops.SeqBatchTensors(
        cu_seqlens=torch.tensor([0, seq], dtype=torch.int32, device=dev),
        block_tables=torch.zeros(1, 1, dtype=torch.int32, device=dev),
        max_seq_len=seq,
        positions=pos,
    )
    chunks_k = [_rank_chunks(fk) for fk, _ in factors]
    chunks_v = [_rank_chunks(fv) for _, fv in factors]
    n_chunks = max(max(len(c) for c in chunks_k), max(len(c) for c in chunks_v))
    st = ops.status_word(dev)
    for ci in range(n_chunks):
        fks = [c[ci] if ci < len(c) else None for c in chunks_k]
        fvs = [c[ci] if ci < len(c) else None for c in chunks_v]
        rk = max((f[0].shape[0] for f in fks if f is not None), default=0)
        rv = max((f[0].shape[0] for f in fvs if f is not None), default=0)
        geom = ops.exact_geometry(d, n_kv, hd, torch.float16, rk, rv)
        ref = next(f for f in fks + fvs if f is not None) if (rk or rv) else None
        dt = torch.float32
        def stack(which, idx, rank, rows, cols):
            mats = []
            for f in which:
                m = torch.zeros(rows, cols, dtype=dt, device=dev)
                if f is not None:
                    src = f[idx].to(device=dev, dtype=dt)
                    m[: src.shape[0], : src.shape[1]] = src
                mats.append(m)
            return torch.stack(mats)
        d_kv = n_kv * hd
        a_k = stack(fks, 0, rk, rk, d) if rk else None
        b_k = stack(fks, 1, rk, d_kv, rk) if rk else None
        a_v = stack(fvs, 0, rv, rv, d) if rv else None
        b_v = stack(fvs, 1, rv, d_kv, rv) if rv else None
        # per-layer scales are folded into B so one launch serves layers with different scales
        if rk:
            for l, f in enumerate(fks):
                if f is not None:
                    b_k[l] *= float(f[2])
        if rv:
            for l, f in enumerate(fvs):
                if f is not None:
                    b_v[l] *= float(f[2])
        packed = ops.pack_factors(geom, a_k, b_k, a_v, b_v, 1.0, 1.0) if ref is not None else None
        if packed is None:
            # no factors at all: only zeros are written (store) or nothing (accumulate)
            if not (ci == 0 and not accumulate_first):
                continue
            for o in out_k + out_v:
                o.zero_()
            continue
        ops.exact_patch_paged(
            geom, xq, packed, [_dense_pages(o) for o in out_k], [_dense_pages(o) for o in out_v], seqs,
            x_scale=xs, apply_norm=False, rope_cos=cos, rope_sin=sin,
            accumulate=accumulate_first or ci > 0, status=st,
        )


def exact_kv_patch(x_normed: Tensor, layer, *, n_kv_heads: int, head_dim: int, rope=None,
                   positions: Tensor | None = None) -> LowRankKVPatch:
    """Exact dK/dV given the true input activations of this layer's k/v projections.

    ``dK = RoPE(scale_k * (x @ A_k^T) @ B_k^T)`` (no RoPE when ``rope`` is None),
    ``dV = scale_v * (x @ A_v^T) @ B_v^T``; a missing projection gives zeros.
    """
    ops._require_cuda(x_normed)
    seq = x_normed.shape[0]
    fk, fv = kv_factors(layer)
    dk = torch.empty(seq, n_kv_heads, head_dim, dtype=torch.float32, device=x_normed.device)
    dv = torch.empty_like(dk)
    if seq:
        _dense_delta([x_normed], [(fk, fv)], n_kv_heads, head_dim, rope, positions, [dk], [dv],
                     accumulate_first=False)
    return LowRankKVPatch(layer_idx=layer.layer_idx, k_codes=None, k_basis=None, v_codes=None,
                          v_basis=None, k_dense=dk, v_dense=dv)


def zeroth_order_patches(hidden_normed: dict[int, Tensor], delta, *, n_kv_heads: int, head_dim: int,
                         rope=None, positions: Tensor | None = None) -> dict[int, LowRankKVPatch]:
    """Adapter path on cached activations at every modified layer, batched: layers that
    share a sequence length go through one launch."""
    items = [(idx, layer, hidden_normed.get(idx)) for idx, layer in delta.layers.items()]
    items = [(i, ly, x) for i, ly, x in items if x is not None]
    out: dict[int, LowRankKVPatch] = {}
    groups: dict[tuple, list] = {}
    for idx, layer, x in items:
        groups.setdefault((tuple(x.shape), x.device), []).append((idx, layer, x))
    for (_, dev), members in groups.items():
        seq = members[0][2].shape[0]
        dks = [torch.empty(seq, n_kv_heads, head_dim, dtype=torch.float32, device=dev) for _ in members]
        dvs = [torch.empty_like(t) for t in dks]
        for start in range(0, len(members), L.DKV_MAX_LAYERS):
            part = slice(start, start + L.DKV_MAX_LAYERS)
            if seq:
                _dense_delta([m[2] for m in members[part]], [kv_factors(m[1]) for m in members[part]],
                             n_kv_heads, head_dim, rope, positions, dks[part], dvs[part], accumulate_first=False)
        for (idx, layer, _), dk, dv in zip(members, dks, dvs):
            out[idx] = LowRankKVPatch(layer_idx=layer.layer_idx, k_codes=None, k_basis=None, v_codes=None,
                                      v_basis=None, k_dense=dk, v_dense=dv)
    return out


def materialize_codes(codes: Tensor, basis: Tensor, n_kv_heads: int, head_dim: int) -> Tensor:
    """``codes [seq, r] @ basis[d_kv, r]^T`` as ``[seq, n_kv, hd]`` fp32 — the expand half of
    the fused kernel (identity A, the codes as activations, no RoPE)."""
    ops._require_cuda(codes, basis)
    seq, r = codes.shape
    out = torch.empty(seq, n_kv_heads, head_dim, dtype=torch.float32, device=codes.device)
    if seq == 0:
        return out
    eye = torch.eye(r, dtype=torch.float32, device=codes.device)
    _dense_delta([codes.float()], [(None, (eye, basis.float(), 1.0))], n_kv_heads, head_dim, None, None,
                 [torch.empty_like(out)], [out], accumulate_first=False)
    return out


def _add_dense(dst: Tensor, delta: Tensor) -> None:
    seq = dst.shape[0]
    seqs = ops.SeqBatchTensors(
        cu_seqlens=torch.tensor([0, seq], dtype=torch.int32, device=dst.device),
        block_tables=torch.zeros(1, 1, dtype=torch.int32, device=dst.device),
        max_seq_len=seq,
    )
    ops.scatter_paged(delta, dst.unsqueeze(0), seqs)


def apply_layer_patches(kv, patches: dict[int, LowRankKVPatch]) -> KVCache:
    """Clone ``kv`` and add every layer's materialised dK / dV (compose.py:29-34)."""
    out = kv.clone() if hasattr(kv, "clone") else KVCache(kv.k.clone(), kv.v.clone(), kv.version)
    n_kv, hd = out.k.shape[2], out.k.shape[3]
    for idx, p in patches.items():
        dk, dv = p.materialize(n_kv, hd)
        if out.k.shape[1]:
            _add_dense(out.k[idx], dk)
            _add_dense(out.v[idx], dv)
    return out


def apply_layer_patches_(kv, patches: dict[int, LowRankKVPatch]):
    """``apply_layer_patches`` without the clone: every layer's dK / dV is added to ``kv`` in
    place (dense parts by the paged add, codes @ basis by the fused kernel's expand half, which
    accumulates straight into the cache layer).  Returns ``kv``."""
    n_kv, hd = kv.k.shape[2], kv.k.shape[3]
    seq = kv.k.shape[1]
    if seq == 0:
        return kv
    for idx, p in patches.items():
        for dst, dense, codes, basis in ((kv.k[idx], p.k_dense, p.k_codes, p.k_basis),
                                         (kv.v[idx], p.v_dense, p.v_codes, p.v_basis)):
            if dense is not None:
                _add_dense(dst, dense)
            elif codes is not None and basis is not None:
                r = codes.shape[1]
                eye = torch.eye(r, dtype=torch.float32, device=dst.device)
                scratch = torch.empty_like(dst)
                _dense_delta([codes.float()], [(None, (eye, basis.float(), 1.0))], n_kv, hd, None, None,
                             [scratch], [dst], accumulate_first=True)
            else:
                raise ValueError("patch is empty")
    return kv


def replay(base, chain, *, inplace: bool = False):
    """The engine's STRICT-hit replay (engine.py:205-210) — base plus every stage of the patch
    chain — with one copy of the base at most (none with ``inplace=True``) instead of a clone
    per stage; each stage's patches are added in place."""
    kv = base if inplace else (base.clone() if hasattr(base, "clone") else KVCache(base.k.clone(), base.v.clone(),
                                                                                   base.version))
    for applied in chain:
        apply_layer_patches_(kv, applied.layer_patches)
        kv.version = applied.target
    return kv
