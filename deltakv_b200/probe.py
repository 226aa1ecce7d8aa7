"""Probe scoring, selection, the CacheBlend residual gate and the probe route per layer.

Drop-ins for src/deltakv/patches/probe.py (same names, arguments and results):

* ``lora_activation_scores`` (patches/exact.py:111-115) and ``weight_axis_scores``
  (probe.py:30-47): per-token ``||s x A^T||`` on the GPU (``dkv_lora_scores``), summed over a
  layer's projections;
* ``select_probes`` (probe.py:14-27): top-b tokens, always token 0 — a device ``topk``;
* ``residual_gate`` (probe.py:85-109): per-token residual estimates by ``dkv_row_diff_norms``,
  then the threshold and the capped top-k;
* ``apply_probe_to_cache`` (probe.py:112-165): per layer the subspace correction of K (basis
  from the probe residual) and V (the adapter's LoRA B) with this package's kernels, the gate on
  ``probe_layers``, and the per-layer dense patches.
"""

from __future__ import annotations

import ctypes as C

import torch
from torch import Tensor

from deltakv_b200 import _lib as L
from deltakv_b200 import ops
from deltakv_b200.subspace import subspace_correct_batched
from deltakv_b200.types import KVCache, LowRankKVPatch


def _rows2(t: Tensor) -> Tensor:
    r = t.reshape(t.shape[0], -1)
    return r if r.stride(-1) == 1 else r.contiguous()


def lora_activation_scores(x_normed: Tensor, fac) -> Tensor:
    """Per-token score ``||x A^T|| * scale`` — tokens that fire the adapter the hardest."""
    if fac is None or int(x_normed.shape[-1]) != int(fac.A.shape[1]):
        return x_normed.new_zeros(x_normed.shape[0])
    ops._require_cuda(x_normed)
    x = _rows2(x_normed)
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        x = x.float()
    a = fac.A.to(device=x.device, dtype=torch.float32).contiguous()
    out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    rc = L.lib().dkv_lora_scores(x.data_ptr(), ops.dkv_dtype(x.dtype), x.shape[0], x.shape[1], x.stride(0),
                                 a.data_ptr(), a.shape[0], float(getattr(fac, "scale", 1.0)), out.data_ptr(), 0,
                                 ops.stream_ptr())
    L.check(rc, "dkv_lora_scores")
    return out.to(x_normed.dtype) if x_normed.dtype != torch.float32 else out


def weight_axis_scores(x_normed: Tensor, delta, layer_idx: int = 0) -> Tensor:
    """Tokens that fire LoRA/edit factors the hardest at the first modified layer."""
    layers = delta.layers
    first = getattr(delta, "first_modified_layer", min(layers) if layers else 0)
    layer = layers.get(layer_idx) or layers.get(first)
    if layer is None:
        return x_normed.new_ones(x_normed.shape[0])
    acc = x_normed.new_zeros(x_normed.shape[0], dtype=torch.float32)
    in_dim = int(x_normed.shape[-1])
    projections = getattr(layer, "projections", None)
    facs = projections.values() if projections is not None else []
    for fac in facs:
        if int(fac.A.shape[1]) != in_dim:
            continue
        acc = acc + lora_activation_scores(x_normed, fac).float()
    if float(acc.max()) <= 0:
        return x_normed.new_ones(x_normed.shape[0])
    return acc.to(x_normed.dtype)


def select_probes(scores: Tensor, ratio: float, min_tokens: int = 4, max_ratio: float = 0.5) -> Tensor:
    """Return indices of the top-b tokens. Always includes 0 (BOS/anchor)."""
    n = int(scores.numel())
    b = int(max(min_tokens, round(ratio * n)))
    b = min(b, max(1, int(max_ratio * n)), n)
    top = torch.topk(scores, k=b, largest=True).indices
    if not bool((top == 0).any()):
        top = torch.cat([scores.new_zeros(1, dtype=torch.long), top[:-1]])
    return torch.unique(top.sort().values)


def _diff_norms(a: Tensor, b: Tensor, rows: Tensor | None) -> Tensor:
    a2, b2 = _rows2(a), _rows2(b)
    if a2.dtype != b2.dtype or a2.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        a2, b2 = a2.float(), b2.float()
    idx = None if rows is None else rows.to(device=a2.device, dtype=torch.int32).contiguous()
    n_out = a2.shape[0] if idx is None else idx.numel()
    out = torch.empty(n_out, dtype=torch.float32, device=a2.device)
    st = ops.status_word(a2.device)
    rc = L.lib().dkv_row_diff_norms(a2.data_ptr(), b2.data_ptr(), ops.dkv_dtype(a2.dtype), a2.shape[0], a2.shape[1],
                                    a2.stride(0), b2.stride(0), ops.ptr(idx), n_out, out.data_ptr(), st.ptr,
                                    ops.stream_ptr())
    L.check(rc, "dkv_row_diff_norms")
    return out


def residual_gate(reused: Tensor, corrected: Tensor, fresh_probe: Tensor, probe_index: Tensor, threshold: float,
                  max_ratio: float) -> Tensor:
    """CacheBlend-style extra recompute: tokens whose estimated residual stays large relative
    to the probes' residual scale, capped at ``max_ratio * seq`` tokens in all."""
    ops._require_cuda(reused, corrected, fresh_probe)
    seq = reused.shape[0]
    idx = probe_index.to(device=reused.device, dtype=torch.long).reshape(-1)
    est = _diff_norms(corrected, reused, None)
    probe_scale = _diff_norms(fresh_probe, reused, idx % max(seq, 1) if idx.numel() else idx)
    scale = probe_scale.mean().clamp_min(1e-8) if probe_scale.numel() else est.new_tensor(1e-8)
    relative = est / scale
    extra = (relative > threshold).nonzero(as_tuple=False).view(-1)
    cap = max(0, int(max_ratio * seq) - int(idx.numel()))
    if extra.numel() > cap:
        extra = extra[relative[extra].topk(cap).indices]
    return extra


def bases_for_layer(layer) -> tuple[Tensor | None, Tensor | None]:
    """LoRA ``B`` for k_proj / v_proj, or None if that map has no delta (subspace.py:109-119)."""
    if layer is None:
        return None, None
    k_fac, v_fac = layer.get("k_proj"), layer.get("v_proj")
    return (k_fac.B if k_fac is not None else None), (v_fac.B if v_fac is not None else None)


def _k_bases(kv, fresh_layers: dict, probe_index: Tensor, layer_deltas: dict | None, subspace_rank: int,
             skip_layers: set | None) -> dict[int, Tensor]:
    """The K path's basis of every layer (``svd_basis`` of the probe residual at rank
    ``B_k``'s width, subspace.py:91-93), all layers of one rank in one batched
    :func:`~deltakv_b200.subspace.topr_basis` call.  Layers are independent, so the residuals
    can be formed before any layer is corrected."""
    from deltakv_b200.subspace import probe_residual, topr_basis

    groups: dict[int, list[int]] = {}
    idx = None
    for l, (fk, _) in fresh_layers.items():
        if skip_layers is not None and l in skip_layers:
            continue
        seq = int(kv.k[l].shape[0])
        if idx is None:
            idx = probe_index.to(device=fk.device, dtype=torch.int64).reshape(-1)
            if idx.numel() < 2:
                return {}
            lo, hi = int(idx.min()), int(idx.max())
            if lo < -seq or hi >= seq:
                return {}  # subspace_correct raises the reference's IndexError for this layer
            idx = torch.where(idx < 0, idx + seq, idx).to(torch.int32).contiguous()
        k_b, _ = bases_for_layer(None if layer_deltas is None else layer_deltas.get(l))
        k_rank = int(k_b.shape[1]) if k_b is not None else subspace_rank
        d = int(kv.k[l][0].numel())
        groups.setdefault(min(k_rank, max(1, idx.numel() - 1), d), []).append(l)
    out: dict[int, Tensor] = {}
    for r, ls in groups.items():
        res = torch.stack([probe_residual(_rows2(kv.k[l]), _rows2(fresh_layers[l][0]).to(kv.k[l].dtype), idx)
                           for l in ls])
        bases = topr_basis(res, r)
        for j, l in enumerate(ls):
            out[l] = bases[j]
    return out


def apply_probe_to_cache(kv, fresh_layers: dict, probe_index: Tensor, blend_threshold: float = 0.15,
                         blend_max_ratio: float = 0.40, *, layer_deltas: dict | None = None, subspace_rank: int = 8,
                         probe_layers: set | None = None, skip_layers: set | None = None):
    """Correct cached KV with a rank-r subspace shift plus residual mu, per layer.

    V uses the adapter's LoRA ``B`` as the exact column space; K (RoPE'd) the SVD of the probe
    residual at rank ``B_k``'s width (or ``subspace_rank``).  Layers in ``probe_layers`` (all
    when None) also run the residual gate, whose extra tokens take the fresh value.  Returns
    ``(corrected KVCache, {layer: dense patch}, extra token indices)``.
    """
    out = kv.clone() if hasattr(kv, "clone") else KVCache(kv.k.clone(), kv.v.clone(), kv.version)
    patches: dict[int, LowRankKVPatch] = {}
    extra_all: list[Tensor] = []
    k_bases = _k_bases(out, fresh_layers, probe_index, layer_deltas, subspace_rank, skip_layers)
    # every layer's K and V correction in one batched call (each reads only its own layer)
    layers = [l for l in fresh_layers if skip_layers is None or l not in skip_layers]
    probs = []
    for l in layers:
        fk, fv = fresh_layers[l]
        layer = None if layer_deltas is None else layer_deltas.get(l)
        k_b, v_b = bases_for_layer(layer)
        k_rank = int(k_b.shape[1]) if k_b is not None else subspace_rank
        probs.append(dict(reused=out.k[l], fresh=fk, probe_index=probe_index, basis=k_bases.get(l), rank=k_rank))
        probs.append(dict(reused=out.v[l], fresh=fv, probe_index=probe_index, basis=v_b, rank=subspace_rank))
    corrected = subspace_correct_batched(probs)
    for j, l in enumerate(layers):
        fk, fv = fresh_layers[l]
        rk, rv = out.k[l], out.v[l]
        k_c, v_c = corrected[2 * j][0], corrected[2 * j + 1][0]
        gated = probe_layers is None or l in probe_layers
        if gated:
            extra = residual_gate(rk, k_c, fk, probe_index, blend_threshold, blend_max_ratio)
            if extra.numel():
                k_c[extra] = fk[extra].to(k_c.dtype)
                v_c[extra] = fv[extra].to(v_c.dtype)
                extra_all.append(extra)
        out.k[l] = k_c
        out.v[l] = v_c
        # formed after the layer is overwritten through the views rk / rv, as the reference
        # orders it (probe.py:150-163)
        patches[l] = LowRankKVPatch(layer_idx=l, k_codes=None, k_basis=None, v_codes=None, v_basis=None,
                                    k_dense=k_c - rk, v_dense=v_c - rv)
    extra_idx = (torch.unique(torch.cat(extra_all)) if extra_all
                 else probe_index.new_empty(0, dtype=torch.long))
    return out, patches, extra_idx
