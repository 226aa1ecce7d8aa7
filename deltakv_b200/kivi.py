"""KIVI-style int4 KV caches on the B200 kernels.

K tensors use per-channel groups (32 consecutive tokens of a channel), V tensors per-token
groups (32 consecutive channels); asymmetric min-max with fp16 scale and zero, two codes per
byte.  The reference keeps caches in the model dtype and only fake-quantises them to report
a noise floor (metrics._minmax_quantize, src/deltakv/metrics.py:115-132); this is the stored
counterpart, so a patch can be applied as dequant -> add -> requant in one pass.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
from torch import Tensor

from deltakv_b200 import _lib as L
from deltakv_b200 import ops

GROUP = 32


@dataclass
class KiviTensor:
    """One int4 K or V tensor of ``n_tokens x d``."""

    codes: Tensor  # uint8 [n, d/2]
    scale: Tensor  # fp16, V: [n, d/32], K: [ceil(n/32), d]
    zero: Tensor
    mode: str      # "k" (per channel) or "v" (per token)

    @property
    def n_tokens(self) -> int:
        return int(self.codes.shape[0])

    @property
    def d(self) -> int:
        return int(self.codes.shape[1]) * 2

    @staticmethod
    def empty(n_tokens: int, d: int, mode: str, device) -> "KiviTensor":
        if d % GROUP:
            raise ValueError("d must be a multiple of 32")
        codes = torch.empty(n_tokens, d // 2, dtype=torch.uint8, device=device)
        if mode == "v":
            shape = (n_tokens, d // GROUP)
        elif mode == "k":
            shape = ((n_tokens + GROUP - 1) // GROUP, d)
        else:
            raise ValueError("mode must be 'k' or 'v'")
        return KiviTensor(codes, torch.empty(shape, dtype=torch.float16, device=device),
                          torch.empty(shape, dtype=torch.float16, device=device), mode)

    def desc(self) -> L.KiviCache:
        ops._require_cuda(self.codes, self.scale, self.zero)
        if self.scale.stride() != self.zero.stride() or self.scale.stride(1) != 1 or self.codes.stride(1) != 1:
            raise ValueError("scale/zero must share a row-major layout; codes rows contiguous")
        return L.KiviCache(
            codes=self.codes.data_ptr(), scale=self.scale.data_ptr(), zero=self.zero.data_ptr(),
            code_row_stride=self.codes.stride(0), sz_row_stride=self.scale.stride(0),
            n_tokens=self.n_tokens, d=self.d,
            mode=L.DKV_KIVI_PER_CHANNEL if self.mode == "k" else L.DKV_KIVI_PER_TOKEN,
        )


def _rows(x: Tensor) -> Tensor:
    x2 = x.reshape(x.shape[0], -1)
    return x2 if x2.stride(1) == 1 else x2.contiguous()


def quantize(x: Tensor, mode: str) -> KiviTensor:
    """``x [n, ...]`` (fp32/bf16/f16) -> int4 with the K ("k") or V ("v") grouping."""
    x2 = _rows(x)
    out = KiviTensor.empty(x2.shape[0], x2.shape[1], mode, x2.device)
    desc = out.desc()
    rc = L.lib().dkv_kivi_quantize(x2.data_ptr(), ops.dkv_dtype(x2.dtype), x2.stride(0), C.byref(desc),
                                   ops.stream_ptr())
    L.check(rc, "dkv_kivi_quantize")
    return out


def dequantize(t: KiviTensor, dtype: torch.dtype = torch.float32) -> Tensor:
    out = torch.empty(t.n_tokens, t.d, dtype=dtype, device=t.codes.device)
    desc = t.desc()
    rc = L.lib().dkv_kivi_dequantize(C.byref(desc), out.data_ptr(), ops.dkv_dtype(dtype), out.stride(0),
                                     ops.stream_ptr())
    L.check(rc, "dkv_kivi_dequantize")
    return out


def patch(base: KiviTensor, delta: Tensor | None, out: KiviTensor | None = None) -> KiviTensor:
    """``out = int4(dequant(base) + delta)``; ``out=None`` patches ``base`` in place."""
    out = base if out is None else out
    bd, od = base.desc(), out.desc()
    dptr, ddt, drs = None, 0, 0
    if delta is not None:
        d2 = _rows(delta)
        ops._require_cuda(d2)
        dptr, ddt, drs = d2.data_ptr(), ops.dkv_dtype(d2.dtype), d2.stride(0)
    rc = L.lib().dkv_kivi_patch(C.byref(bd), dptr, ddt, drs, C.byref(od), ops.stream_ptr())
    L.check(rc, "dkv_kivi_patch")
    return out


@dataclass
class SubspaceProblem:
    """One int4 view to correct: a layer's K or V of one adapter.

    ``basis`` ``[d, r]`` is the column space (V: the adapter's LoRA ``B``); ``None`` takes
    the top-``rank`` (at least 1) right singular vectors of the probe residual when there are
    two or more probes, as the reference's K path does (``svd_basis``,
    src/deltakv/patches/subspace.py:37-42, 91-93) — computed for all such problems of a
    call by one batched subspace iteration (:func:`deltakv_b200.subspace.topr_basis`, exact
    SVD where its gap estimate says the iteration is not converged); with fewer probes the
    correction is the mean shift alone.
    ``out=None`` corrects ``base`` in place.
    """

    base: KiviTensor
    fresh: Tensor
    probe_index: Tensor
    basis: Tensor | None = None
    rank: int = 8
    out: KiviTensor | None = None


def probe_residual(base: KiviTensor, fresh: Tensor, probe_index: Tensor, out: Tensor | None = None) -> Tensor:
    """``fresh[P] - dequant(base)[P]`` as fp32 ``[|P|, d]``, read straight from the int4 cache."""
    f = _rows(fresh)
    rows = probe_index.to(device=f.device, dtype=torch.int32).contiguous()
    if out is None:
        out = torch.empty(rows.numel(), base.d, dtype=torch.float32, device=f.device)
    desc = base.desc()
    st = ops.status_word(f.device)
    rc = L.lib().dkv_kivi_probe_residual(C.byref(desc), f.data_ptr(), ops.dkv_dtype(f.dtype), f.stride(0),
                                         rows.data_ptr(), rows.numel(), out.data_ptr(), out.stride(0), st.ptr,
                                         ops.stream_ptr())
    L.check(rc, "dkv_kivi_probe_residual")
    return out


def probe_residuals(bases: list[KiviTensor], freshes: list[Tensor], probe_indices: list[Tensor],
                    out: Tensor | None = None) -> Tensor:
    """:func:`probe_residual` for many caches in one launch: ``out[j] = fresh_j[P_j] -
    dequant(base_j)[P_j]`` as fp32 ``[jobs, |P|, d]`` (every ``P_j`` the same length, every
    fresh the same dtype)."""
    if not bases:
        raise ValueError("no caches")
    fr = [_rows(f) for f in freshes]
    dev = fr[0].device
    conv: dict = {}  # one int32 copy per distinct probe tensor
    rows = []
    for p in probe_indices:
        key = (p.data_ptr(), p.numel(), p.dtype)
        if key not in conv:
            conv[key] = p.to(device=dev, dtype=torch.int32).contiguous()
        rows.append(conv[key])
    m, d = rows[0].numel(), bases[0].d
    if any(r.numel() != m for r in rows) or any(f.dtype != fr[0].dtype for f in fr):
        raise ValueError("probe_residuals: every job needs the same probe count and fresh dtype")
    if out is None:
        out = torch.empty(len(bases), m, d, dtype=torch.float32, device=dev)
    jobs = (L.KiviProbeJob * len(bases))(*[
        L.KiviProbeJob(base=b.desc(), fresh=f.data_ptr(), fresh_row_stride=f.stride(0), rows=r.data_ptr())
        for b, f, r in zip(bases, fr, rows)])
    st = ops.status_word(dev)
    rc = L.lib().dkv_kivi_probe_residual_batched(jobs, len(bases), ops.dkv_dtype(fr[0].dtype), m, out.data_ptr(),
                                                 out.stride(0), out.stride(1), st.ptr, ops.stream_ptr())
    L.check(rc, "dkv_kivi_probe_residual_batched")
    return out


def k_bases(problems: list[SubspaceProblem]) -> dict[int, Tensor]:
    """The K path's bases: for every problem without a basis and with two or more probes, the
    top-``rank`` right singular subspace of its probe residual (``svd_basis``,
    src/deltakv/patches/subspace.py:37-42, 91-93), all problems of one shape in one batched
    subspace iteration (:func:`deltakv_b200.subspace.topr_basis`).  Keyed by problem index."""
    from deltakv_b200 import subspace as dense_sub

    need = {}
    for i, pb in enumerate(problems):
        if pb.basis is None and pb.probe_index.numel() >= 2:
            m, d = pb.probe_index.numel(), pb.base.d
            need.setdefault((m, d, min(int(pb.rank), max(1, m - 1), d), pb.fresh.dtype), []).append(i)
    svd = {}
    for (m, d, r, _), idx in need.items():
        res = probe_residuals([problems[i].base for i in idx], [problems[i].fresh for i in idx],
                              [problems[i].probe_index for i in idx])
        bases = dense_sub.topr_basis(res, r)
        for j, i in enumerate(idx):
            svd[i] = bases[j]
    return svd


def subspace_correct(problems: list[SubspaceProblem], *, stats: bool = False, check: bool = True,
                     bases: dict[int, Tensor] | None = None):
    """Batched subspace correction of int4 caches: one launch per pass for every problem.

    Returns, per problem, ``(out, subspace, orth_mu)`` (the last two ``[d]`` fp32, or None
    unless ``stats``) — the int4 form of ``subspace_correct``'s ``(corrected, subspace,
    orth_mu)``.  ``bases`` (from :func:`k_bases`) skips computing the K bases here.
    """
    if not problems:
        return []
    dev = problems[0].fresh.device
    keep = []  # tensors that must stay alive until the launches are queued
    descs = []
    results = []
    svd = k_bases(problems) if bases is None else bases
    probe_rows: dict = {}  # one int32 copy per distinct probe tensor of the call
    for i, pb in enumerate(problems):
        fresh = _rows(pb.fresh)
        ops._require_cuda(fresh, pb.probe_index)
        n, d = pb.base.n_tokens, pb.base.d
        if fresh.shape != (n, d):
            raise ValueError(f"fresh {tuple(fresh.shape)} does not match the int4 base ({n}, {d})")
        pk = (pb.probe_index.data_ptr(), pb.probe_index.numel(), pb.probe_index.dtype)
        probes = probe_rows.get(pk)
        if probes is None:
            probes = pb.probe_index.to(device=dev, dtype=torch.int32).contiguous()
            probe_rows[pk] = probes
        basis = pb.basis if pb.basis is not None else svd.get(i)  # svd_basis keeps at least rank 1
        if basis is not None:
            if basis.shape[0] != d:
                raise ValueError(f"basis d={basis.shape[0]} != kv d={d}")
            basis = basis.to(device=dev, dtype=torch.float32).contiguous()
            rank = basis.shape[1]
        else:
            rank = 0
        out = pb.out if pb.out is not None else pb.base
        sub = torch.empty(d, dtype=torch.float32, device=dev) if stats else None
        mu = torch.empty(d, dtype=torch.float32, device=dev) if stats else None
        keep += [fresh, probes, basis, sub, mu]
        descs.append(L.KiviSubspaceProblem(
            base=pb.base.desc(), out=out.desc(), fresh=fresh.data_ptr(), fresh_dtype=ops.dkv_dtype(fresh.dtype),
            fresh_row_stride=fresh.stride(0), probe_index=probes.data_ptr(), n_probes=probes.numel(),
            basis=ops.ptr(basis), rank=rank, subspace_out=ops.ptr(sub), orth_mu_out=ops.ptr(mu)))
        results.append((out, sub, mu))
    arr = (L.KiviSubspaceProblem * len(descs))(*descs)
    nbytes = C.c_int64()
    L.check(L.lib().dkv_kivi_subspace_workspace_bytes(arr, len(descs), C.byref(nbytes)),
            "dkv_kivi_subspace_workspace_bytes")
    ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=dev)
    st = ops.status_word(dev)
    rc = L.lib().dkv_kivi_subspace_correct(arr, len(descs), ws.data_ptr(), ws.numel(), st.ptr, ops.stream_ptr())
    L.check(rc, "dkv_kivi_subspace_correct")
    if check:
        st.raise_if_set("kivi.subspace_correct")
    return results


_side_streams: dict[str, torch.cuda.Stream] = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    key = str(device)
    if key not in _side_streams:
        # high priority: the bases' small latency-bound kernels are dispatched ahead of the
        # route's queued CTAs instead of after them
        lo, hi = torch.cuda.Stream.priority_range()
        _side_streams[key] = torch.cuda.Stream(device=device, priority=hi)
    return _side_streams[key]


def subspace_correct_views(views: list[list[SubspaceProblem]], *, stats: bool = False, check: bool = True):
    """:func:`subspace_correct` for several adapter views in turn (the reference's per-view
    ``apply_probe_to_cache`` loop, src/deltakv/patches/probe.py:112-165), with the K bases of
    view v + 1 computed on a side stream while view v's route runs: the bases' small solver
    kernels fill the route's idle SM time; view 0's problems that need no such basis run while
    view 0's bases are computed.  A view that corrects a cache in place is finished before the
    next view's bases read anything.  Returns one result list per view."""
    views = [v for v in views]
    if not views or not any(views):
        return [[] for _ in views]
    dev = next(v for v in views if v)[0].fresh.device
    main = torch.cuda.current_stream(dev)
    side = _side_stream(dev)

    def launch_bases(v: int, after_main: bool):
        if after_main:  # everything queued on main so far happens before these bases
            side.wait_stream(main)
        with torch.cuda.stream(side):
            kb = k_bases(views[v]) if views[v] else {}
        ev = torch.cuda.Event()
        ev.record(side)
        return kb, ev

    def in_place(probs: list[SubspaceProblem]) -> bool:
        return any(pb.out is None or pb.out.codes.data_ptr() == pb.base.codes.data_ptr() for pb in probs)

    # view 0's problems that need no basis from the probe residual (V, whose basis is the
    # adapter's B) go first, so the main stream is busy while view 0's K bases are computed —
    # unless one of their outputs is a cache those bases read
    first = views[0]
    kpos = [i for i, pb in enumerate(first) if pb.basis is None and pb.probe_index.numel() >= 2]
    opos = [i for i in range(len(first)) if i not in set(kpos)]
    reads = {first[i].base.codes.data_ptr() for i in kpos}
    writes = {(first[i].out or first[i].base).codes.data_ptr() for i in opos}
    ahead = {}
    if kpos and opos and not (reads & writes):
        ready = torch.cuda.Event()
        ready.record(main)  # the inputs were produced on main
        ahead = dict(zip(opos, subspace_correct([first[i] for i in opos], stats=stats, check=False, bases={})))
        side.wait_event(ready)
        nxt = launch_bases(0, False)
    else:
        nxt = launch_bases(0, True)  # the inputs were produced on main
    out = []
    for v, probs in enumerate(views):
        kb, ev = nxt
        main.wait_event(ev)
        for t in kb.values():
            t.record_stream(main)
        if v == 0 and ahead:
            rest = subspace_correct([first[i] for i in kpos], stats=stats, check=False,
                                    bases={j: kb[i] for j, i in enumerate(kpos) if i in kb})
            ahead.update(zip(kpos, rest))
            out.append([ahead[i] for i in range(len(first))])
        else:
            out.append(subspace_correct(probs, stats=stats, check=False, bases=kb) if probs else [])
        if v + 1 < len(views):
            nxt = launch_bases(v + 1, in_place(probs))
    if check:
        ops.status_word(dev).raise_if_set("kivi.subspace_correct_views")
    return out

