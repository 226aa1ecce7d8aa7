"""Per-layer measured error of a patch, the KV comparison report, and the cross-rank gather.

``measured_error`` follows src/deltakv/patches/compose.py:147-163: for each layer,
``(||K_p - K_f|| + ||V_p - V_f||) / (||K_f|| + ||V_f|| + 1e-8)`` and the maximum over layers.
``compare_kv`` follows src/deltakv/metrics.py:60-81: per layer and projection the relative L2
``||p - f|| / (||f|| + 1e-8)`` and the cosine, then their max / mean / min over layers.
Here the sums run in one kernel launch per projection over every layer, reading the patched
KV straight from its pages (no gather), and :func:`gather_layer_errors` is the path's only
collective: each rank's per-layer scalars are all-gathered (NCCL over NVLink on GPUs, gloo on
CPU tensors), so no KV crosses GPUs.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Sequence

import torch
from torch import Tensor

from deltakv_b200 import _lib as L
from deltakv_b200 import ops


@dataclass(frozen=True)
class ErrorEstimate:
    """Field names of the reference's ErrorEstimate (src/deltakv/patches/compose.py)."""

    relative_kv_l2: float
    per_layer: tuple[float, ...]
    measured: bool = True
    notes: str = ""


def _error_sums(pages: Sequence[Tensor], fresh: Tensor, seqs: ops.SeqBatchTensors, sums: Tensor,
                status: ops.StatusWord | None, fn: str = "dkv_paged_error_sums") -> None:
    n_layers = len(pages)
    if fresh.ndim != 4 or fresh.shape[0] != n_layers:
        raise ValueError("fresh must be [n_layers, rows, n_kv, head_dim] matching the page list")
    if fresh.stride(3) != 1:
        raise ValueError("fresh rows must be contiguous along head_dim")
    ops._require_cuda(fresh, sums)
    descs = (L.PagedCache * n_layers)(*[ops.paged_desc(p) for p in pages])
    geo = lambda d: (d.dtype, d.block_size, d.n_heads, d.head_dim, d.stride_block, d.stride_slot, d.stride_head)
    if any(geo(d) != geo(descs[0]) for d in descs):
        raise ValueError("every layer's pages must share dtype, shape and strides")
    rc = getattr(L.lib(), fn)(descs, n_layers, fresh.data_ptr(), ops.dkv_dtype(fresh.dtype), fresh.stride(0),
                              fresh.stride(1), fresh.stride(2), C.byref(seqs.struct()), sums.data_ptr(),
                              status.ptr if status else None, ops.stream_ptr())
    L.check(rc, fn)


@dataclass
class LayerKVError:
    """Field names of the reference's LayerKVError (src/deltakv/metrics.py:14-20)."""

    layer: int
    relative_l2_k: float
    relative_l2_v: float
    cosine_k: float
    cosine_v: float


@dataclass
class CompareReport:
    """Field names of the reference's CompareReport (src/deltakv/metrics.py:23-48)."""

    layers: list[LayerKVError]
    max_relative_l2: float
    mean_relative_l2: float
    min_cosine: float
    next_token_kl: float | None = None
    logprob_mae: float | None = None
    logprob_max: float | None = None
    logit_l2: float | None = None
    kivi4_floor: float | None = None
    within_kivi4: bool | None = None

    def as_dict(self) -> dict[str, float | bool | None]:
        return {
            "max_relative_l2": self.max_relative_l2,
            "mean_relative_l2": self.mean_relative_l2,
            "min_cosine": self.min_cosine,
            "next_token_kl": self.next_token_kl,
            "logprob_mae": self.logprob_mae,
            "logprob_max": self.logprob_max,
            "logit_l2": self.logit_l2,
            "kivi4_floor": self.kivi4_floor,
            "within_kivi4": self.within_kivi4,
        }


def _compare_sums(pages: Sequence[Tensor], fresh: Tensor, seqs: ops.SeqBatchTensors, sums: Tensor,
                  status: ops.StatusWord | None) -> None:
    _error_sums(pages, fresh, seqs, sums, status, fn="dkv_paged_compare_sums")


def compare_kv_paged(k_pages: Sequence[Tensor], v_pages: Sequence[Tensor], k_fresh: Tensor, v_fresh: Tensor,
                     seqs: ops.SeqBatchTensors, *, check: bool = False) -> Tensor:
    """Per-layer ``[n_layers, 4]`` (fp64, on the device): relative L2 of K, of V, cosine of K,
    of V — paged K/V against dense fresh K/V ``[n_layers, rows, n_kv, head_dim]``."""
    dev = k_fresh.device
    n_layers = len(k_pages)
    if len(v_pages) != n_layers:
        raise ValueError("k_pages and v_pages must cover the same layers")
    sums = torch.zeros(2, n_layers, 4, dtype=torch.float64, device=dev)
    st = ops.status_word(dev)
    _compare_sums(k_pages, k_fresh, seqs, sums[0], st)
    _compare_sums(v_pages, v_fresh, seqs, sums[1], st)
    if check:
        st.raise_if_set("compare_kv_paged")
    rel = sums[:, :, 0].sqrt() / (sums[:, :, 1].sqrt() + 1e-8)
    cos = sums[:, :, 2] / (sums[:, :, 3] * sums[:, :, 1]).clamp_min(1e-16).sqrt()
    return torch.stack([rel[0], rel[1], cos[0], cos[1]], dim=1)


def compare_kv(patched, fresh) -> CompareReport:
    """Drop-in for ``deltakv.metrics.compare_kv`` on dense CUDA KV caches (``.k`` / ``.v`` of
    shape ``[n_layers, seq, n_kv, head_dim]``): one kernel launch per projection."""
    pk, pv, fk, fv = patched.k, patched.v, fresh.k, fresh.v
    n_layers, seq = pk.shape[0], pk.shape[1]
    if seq == 0:
        rows = [[0.0, 0.0, 0.0, 0.0] for _ in range(n_layers)]
    else:
        seqs = ops.SeqBatchTensors.single(seq, [0], pk.device)
        kp = [pk[l].unsqueeze(0) for l in range(n_layers)]
        vp = [pv[l].unsqueeze(0) for l in range(n_layers)]
        rows = compare_kv_paged(kp, vp, fk, fv, seqs, check=True).tolist()
    layers = [LayerKVError(layer=l, relative_l2_k=r[0], relative_l2_v=r[1], cosine_k=r[2], cosine_v=r[3])
              for l, r in enumerate(rows)]
    rels = [max(x.relative_l2_k, x.relative_l2_v) for x in layers]
    cos = [min(x.cosine_k, x.cosine_v) for x in layers]
    return CompareReport(layers=layers, max_relative_l2=max(rels) if rels else 0.0,
                         mean_relative_l2=float(sum(rels) / max(len(rels), 1)), min_cosine=min(cos) if cos else 1.0)


def measured_error_paged(k_pages: Sequence[Tensor], v_pages: Sequence[Tensor], k_fresh: Tensor, v_fresh: Tensor,
                         seqs: ops.SeqBatchTensors, *, check: bool = False) -> Tensor:
    """Per-layer relative error ``[n_layers]`` (fp64, on the device) of paged K/V against
    dense fresh K/V ``[n_layers, rows, n_kv, head_dim]`` (rows = the tokens of ``seqs``)."""
    dev = k_fresh.device
    n_layers = len(k_pages)
    if len(v_pages) != n_layers:
        raise ValueError("k_pages and v_pages must cover the same layers")
    sums = torch.zeros(2, n_layers, 2, dtype=torch.float64, device=dev)
    st = ops.status_word(dev)
    _error_sums(k_pages, k_fresh, seqs, sums[0], st)
    _error_sums(v_pages, v_fresh, seqs, sums[1], st)
    if check:
        st.raise_if_set("measured_error_paged")
    num = sums[0, :, 0].sqrt() + sums[1, :, 0].sqrt()
    den = sums[0, :, 1].sqrt() + sums[1, :, 1].sqrt() + 1e-8
    return num / den


def measured_error(patched, fresh) -> ErrorEstimate:
    """Drop-in for ``deltakv.patches.compose.measured_error`` on dense CUDA KV caches
    (``.k`` / ``.v`` of shape ``[n_layers, seq, n_kv, head_dim]``)."""
    pk, pv, fk, fv = patched.k, patched.v, fresh.k, fresh.v
    n_layers, seq, n_kv, hd = pk.shape
    if seq == 0:
        per = [0.0] * n_layers
        return ErrorEstimate(relative_kv_l2=0.0, per_layer=tuple(per))
    dev = pk.device
    # each layer's dense [seq, n_kv, hd] viewed as one block of `seq` slots
    seqs = ops.SeqBatchTensors.single(seq, [0], dev)
    kp = [pk[l].unsqueeze(0) for l in range(n_layers)]
    vp = [pv[l].unsqueeze(0) for l in range(n_layers)]
    per = measured_error_paged(kp, vp, fk, fv, seqs, check=True).tolist()
    return ErrorEstimate(relative_kv_l2=float(max(per)) if per else 0.0, per_layer=tuple(per))


def gather_layer_errors(local: Tensor, group=None) -> Tensor:
    """All-gather every rank's per-layer error scalars: ``[n_local]`` -> ``[world, n_local]``.

    One ``all_gather_into_tensor`` on the default (or given) process group: NCCL when
    ``local`` is on a GPU, gloo for CPU tensors.  Every rank must pass the same ``n_local``
    (pad with NaN for layers a rank does not hold).
    """
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return local.reshape(1, -1).clone()
    world = dist.get_world_size(group)
    flat = local.reshape(-1).contiguous()
    out = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(out, flat, group=group)
    return out.view(world, -1)


def gather_sharded_layer_errors(local: Tensor, layer_ids: Sequence[int], n_layers: int, group=None) -> Tensor:
    """The full ``[n_layers]`` per-layer error list (the ``per_layer`` of
    src/deltakv/patches/compose.py:147-163) when the layers are split across ranks.

    Each rank passes the errors of its own layers (``local[i]`` belongs to layer
    ``layer_ids[i]``); the layer sets of the ranks must be disjoint and together cover
    ``0..n_layers-1``.  One ``all_gather_into_tensor`` of ``[n_layers]`` vectors (NaN where a
    rank holds no layer) on the default or given process group; every rank gets the list.
    """
    import torch.distributed as dist

    ids = torch.as_tensor(list(layer_ids), dtype=torch.long, device=local.device)
    if ids.numel() != local.numel():
        raise ValueError("one error per layer id")
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= n_layers):
        raise ValueError(f"layer ids must lie in [0, {n_layers})")
    mine = torch.full((n_layers,), float("nan"), dtype=local.dtype, device=local.device)
    mine[ids] = local.reshape(-1)
    every = gather_layer_errors(mine, group) if dist.is_available() and dist.is_initialized() else mine[None]
    held = (~torch.isnan(every)).sum(0)
    if not bool((held == 1).all()):
        raise ValueError("the ranks' layer sets must be disjoint and cover every layer")
    return torch.nan_to_num(every, nan=0.0).sum(0)
