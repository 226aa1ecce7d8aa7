"""Analytic route (Route A): first-order propagation of the hidden-state change through the
stack, emitting per-layer dense ΔK / ΔV.

Drop-ins for src/deltakv/patches/analytic.py (same names, arguments and results) and for the
engine's per-layer loop ``DeltaKVEngine._analytic_patches`` (src/deltakv/engine.py:377-432):

* ``rmsnorm_first_order`` (analytic.py:245-262) — ``dkv_rmsnorm_first_order``, one warp per row;
* ``attention_first_order`` (analytic.py:38-95) — the q/k/v/o projections and the LoRA terms
  are plain library GEMMs; RoPE is ``dkv_rope_rows``; the O(n^2) core (scores, softmax, its
  Jacobian against dS, the two context products) is ``dkv_attn_first_order``, which never
  materialises the [H, n, n] matrices, so the ``attn_probs`` the reference returns as its
  fourth value (unused by its engine) is ``None`` unless ``return_attn=True`` asks for it;
* ``mlp_first_order`` (analytic.py:108-138) — gate/up/down GEMMs and ``dkv_swiglu_first_order``;
* ``rank_truncate`` (analytic.py:14-22) — the best rank-r approximation from the top-r right
  singular subspace (fp64 Gram matrix + eigensolver); ``codes @ basis.T`` equals the
  reference's, the factors themselves may differ by a rotation within the subspace;
* ``analytic_patches`` — the engine loop, with ``model`` / ``config`` objects shaped like the
  reference's (``cfg``, ``blocks``, ``rope``; ``hidden_stride``, ``propagator_rank``).

All arithmetic is fp32 (the reference's model dtype for its toy), on the device.
"""

from __future__ import annotations

import time
import weakref

import torch
from torch import Tensor

from deltakv_b200 import _lib as L
from deltakv_b200 import ops
from deltakv_b200.rope import half_tables, max_positions
from deltakv_b200.types import LowRankKVPatch


def _f32(t: Tensor) -> Tensor:
    t = t.float()
    return t if t.is_contiguous() else t.contiguous()


_fused_cache: dict[tuple, tuple] = {}


def _fused_rows(ws: tuple, device: torch.device) -> Tensor:
    """``cat([w.float() for w in ws], 0)`` on ``device``, made once per set of weight tensors
    (the entry holds weak references: a different or modified tensor misses)."""
    key = tuple(id(w) for w in ws) + (str(device),)
    hit = _fused_cache.get(key)
    if hit is not None:
        refs, versions, fused = hit
        if all(r() is w for r, w in zip(refs, ws)) and versions == tuple(w._version for w in ws):
            return fused
    if len(_fused_cache) >= 512:
        _fused_cache.clear()
    fused = torch.cat([_f32(w.to(device)) for w in ws], dim=0)
    torch.cuda.current_stream(device).synchronize()  # once per weight set: usable from any stream
    _fused_cache[key] = (tuple(weakref.ref(w) for w in ws), tuple(w._version for w in ws), fused)
    return fused


def rmsnorm_first_order(x: Tensor, dx: Tensor, weight: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    """RMSNorm(x) and its first-order image under Δx (rows of ``[..., d]``)."""
    ops._require_cuda(x, dx)
    shape = x.shape
    d = int(shape[-1])
    x2, dx2 = _f32(x).reshape(-1, d), _f32(dx).reshape(-1, d)
    w = _f32(weight.to(x2.device))
    y, dy = torch.empty_like(x2), torch.empty_like(x2)
    rc = L.lib().dkv_rmsnorm_first_order(x2.data_ptr(), dx2.data_ptr(), w.data_ptr(), float(eps), x2.shape[0], d,
                                         x2.stride(0), dx2.stride(0), y.data_ptr(), dy.data_ptr(), y.stride(0),
                                         dy.stride(0), ops.stream_ptr())
    L.check(rc, "dkv_rmsnorm_first_order")
    return y.view(shape), dy.view(shape)


def softmax_jacobian_product(attn: Tensor, d_scores: Tensor) -> Tensor:
    """``ΔA = J_softmax(A)[ΔS]`` row-wise: ``a ⊙ (δ − ⟨a, δ⟩)`` for materialised matrices (the
    fused attention core applies it without forming them)."""
    centered = d_scores - (attn * d_scores).sum(dim=-1, keepdim=True)
    return attn * centered


def silu(x: Tensor) -> Tensor:
    return x * torch.sigmoid(x)


def silu_grad(x: Tensor) -> Tensor:
    s = torch.sigmoid(x)
    return s + x * s * (1.0 - s)


def _apply(fac, x: Tensor) -> Tensor:
    """``LowRankFactors.apply``: ``(scale * x A^T) B^T`` (factors.py:61-67)."""
    a = fac.A.to(device=x.device, dtype=torch.float32)
    b = fac.B.to(device=x.device, dtype=torch.float32)
    return (float(getattr(fac, "scale", 1.0)) * (x @ a.t())) @ b.t()


def _rope_(x: Tensor, rope) -> None:
    """In-place RoPE at positions 0..n-1 of an fp32 ``[n, heads, head_dim]`` whose rows hold
    ``heads x head_dim`` contiguous values (any row stride)."""
    n, heads, hd = x.shape
    if n == 0:
        return
    cos, sin = half_tables(rope, x.device)
    rc = L.lib().dkv_rope_rows(x.data_ptr(), n, heads, hd, x.stride(0), cos.data_ptr(), sin.data_ptr(),
                               min(max_positions(rope), cos.shape[0]), ops.stream_ptr())
    L.check(rc, "dkv_rope_rows")


def attention_core(q: Tensor, dq: Tensor, k: Tensor, dk: Tensor, v: Tensor, dv: Tensor, *,
                   want_ctx: bool) -> tuple[Tensor | None, Tensor]:
    """``(ctx, dctx)`` ``[n, H, hd]`` fp32 of the causal first-order attention (see module)."""
    n, H, hd = q.shape
    Hkv = k.shape[1]
    tensors = [q, dq, k, dk, v, dv]
    dt = q.dtype if all(t.dtype == q.dtype for t in tensors) else torch.float32
    q, dq, k, dk, v, dv = [t.to(dt).contiguous() for t in tensors]
    dctx = torch.empty(n, H, hd, dtype=torch.float32, device=q.device)
    ctx = torch.empty_like(dctx) if want_ctx else None
    rc = L.lib().dkv_attn_first_order(q.data_ptr(), dq.data_ptr(), H * hd, k.data_ptr(), dk.data_ptr(), v.data_ptr(),
                                      dv.data_ptr(), Hkv * hd, ops.dkv_dtype(dt), n, H, Hkv, hd, float(hd) ** -0.5,
                                      ops.ptr(ctx), dctx.data_ptr(), H * hd, ops.stream_ptr())
    L.check(rc, "dkv_attn_first_order")
    return ctx, dctx


def _attention_core_views(q: Tensor, dq: Tensor, k: Tensor, dk: Tensor, v: Tensor, dv: Tensor, *,
                          want_ctx: bool) -> tuple[Tensor | None, Tensor]:
    """:func:`attention_core` on fp32 ``[n, heads, head_dim]`` views with dense rows (head
    stride ``head_dim``) that share one row stride per group (q, dq / k, dk, v, dv)."""
    n, H, hd = q.shape
    Hkv = k.shape[1]
    grp_q, grp_kv = (q, dq), (k, dk, v, dv)
    ok = all(t.dtype == torch.float32 and t.stride(2) == 1 and t.stride(1) == hd for t in grp_q + grp_kv)
    ok = ok and dq.stride(0) == q.stride(0) and all(t.stride(0) == k.stride(0) for t in grp_kv)
    if not ok:
        return attention_core(q, dq, k, dk, v, dv, want_ctx=want_ctx)
    dctx = torch.empty(n, H, hd, dtype=torch.float32, device=q.device)
    ctx = torch.empty_like(dctx) if want_ctx else None
    rc = L.lib().dkv_attn_first_order(q.data_ptr(), dq.data_ptr(), q.stride(0), k.data_ptr(), dk.data_ptr(),
                                      v.data_ptr(), dv.data_ptr(), k.stride(0), ops.dkv_dtype(torch.float32), n, H,
                                      Hkv, hd, float(hd) ** -0.5, ops.ptr(ctx), dctx.data_ptr(), H * hd,
                                      ops.stream_ptr())
    L.check(rc, "dkv_attn_first_order")
    return ctx, dctx


def attention_first_order(x: Tensor, dx: Tensor, q_w: Tensor, k_w: Tensor, v_w: Tensor, o_w: Tensor, layer, *,
                          n_heads: int, n_kv_heads: int, head_dim: int, rope, causal_mask: Tensor | None = None,
                          base_weights: bool = False, return_attn: bool = False):
    """``(Δh_attn, ΔK, ΔV, attn_probs)`` for one block (analytic.py:38-95).  ``causal_mask``
    is accepted for signature compatibility; the core applies the causal mask itself."""
    ops._require_cuda(x, dx)
    n = int(x.shape[0])
    xf, dxf = _f32(x), _f32(dx)
    dev = xf.device
    w_qkv = _fused_rows((q_w, k_w, v_w), dev)
    dq_o, dk_o = n_heads * head_dim, n_kv_heads * head_dim
    both = torch.cat([xf, dxf], dim=0) @ w_qkv.t()  # one GEMM for the base and the first-order terms
    base, delta = both[:n], both[n:]
    # [n, heads, head_dim] views into the product (row stride = its width): RoPE and the core
    # take row strides, so nothing is copied out
    q = base[:, :dq_o].view(n, n_heads, head_dim)
    k = base[:, dq_o:dq_o + dk_o].view(n, n_kv_heads, head_dim)
    v = base[:, dq_o + dk_o:].view(n, n_kv_heads, head_dim)
    dq = delta[:, :dq_o].view(n, n_heads, head_dim)
    dk = delta[:, dq_o:dq_o + dk_o].view(n, n_kv_heads, head_dim)
    dv = delta[:, dq_o + dk_o:].view(n, n_kv_heads, head_dim)
    if layer is not None:
        for t, name, heads in ((dq, "q_proj", n_heads), (dk, "k_proj", n_kv_heads), (dv, "v_proj", n_kv_heads)):
            fac = layer.get(name)
            if fac is None:
                continue
            t += _apply(fac, xf).view(n, heads, head_dim)
            if base_weights:
                t += _apply(fac, dxf).view(n, heads, head_dim)
    for t in (q, k, dq, dk):
        _rope_(t, rope)
    o_fac = layer.get("o_proj") if layer is not None else None
    ctx, dctx = _attention_core_views(q, dq, k, dk, v, dv, want_ctx=o_fac is not None or return_attn)
    dh = dctx.reshape(n, -1) @ _f32(o_w.to(dev)).t()
    if o_fac is not None:
        dh = dh + _apply(o_fac, ctx.reshape(n, -1))
    dk, dv = dk.contiguous(), dv.contiguous()  # the patch tensors own their storage
    attn = None
    if return_attn:
        rep = n_heads // n_kv_heads
        kf = k.repeat_interleave(rep, dim=1)
        scores = torch.einsum("qhd,khd->hqk", q, kf) * head_dim ** -0.5
        mask = torch.triu(torch.full((n, n), float("-inf"), device=dev), diagonal=1)
        attn = torch.softmax(scores + mask, dim=-1)
    return dh, dk, dv, attn


def mlp_first_order(x: Tensor, dx: Tensor, gate_w: Tensor, up_w: Tensor, down_w: Tensor, layer,
                    base_weights: bool = False) -> Tensor:
    """First-order SwiGLU block (analytic.py:108-138)."""
    ops._require_cuda(x, dx)
    n = int(x.shape[0])
    xf, dxf = _f32(x), _f32(dx)
    dev = xf.device
    ff = int(gate_w.shape[0])
    both = torch.cat([xf, dxf], dim=0) @ _fused_rows((gate_w, up_w), dev).t()
    g, u = both[:n, :ff].contiguous(), both[:n, ff:].contiguous()
    dg, du = both[n:, :ff].contiguous(), both[n:, ff:].contiguous()
    if layer is not None:
        for t, name in ((dg, "gate_proj"), (du, "up_proj")):
            fac = layer.get(name)
            if fac is None:
                continue
            t += _apply(fac, xf)
            if base_weights:
                t += _apply(fac, dxf)
    h, dh = torch.empty_like(g), torch.empty_like(g)
    rc = L.lib().dkv_swiglu_first_order(g.data_ptr(), u.data_ptr(), dg.data_ptr(), du.data_ptr(), g.numel(),
                                        h.data_ptr(), dh.data_ptr(), ops.stream_ptr())
    L.check(rc, "dkv_swiglu_first_order")
    y = dh @ _f32(down_w.to(dev)).t()
    if layer is not None and layer.get("down_proj") is not None:
        y = y + _apply(layer.get("down_proj"), h)
    return y


def rank_truncate(delta: Tensor, rank: int) -> tuple[Tensor, Tensor]:
    """Δ ≈ codes @ basis.T with ``codes [n, r]``, ``basis [d, r]`` (the best rank-r
    approximation, analytic.py:14-22).  The basis is the top-r subspace of the fp64 Gram
    matrix ΔᵀΔ from :func:`deltakv_b200.subspace.gram_topr_basis` (device subspace iteration
    and Rayleigh-Ritz, accepted at an estimated 1e-6 of ‖Δ‖ — the reference's fp32 SVD is
    itself determined only to ~1e-5 where, as for the propagated ΔX, the singular values at
    the cut differ by ~1 % — else the exact eigensolver)."""
    from deltakv_b200.subspace import gram_topr_basis

    ops._require_cuda(delta)
    flat = delta.reshape(delta.shape[0], -1).float()
    r = max(1, min(int(rank), *flat.shape))
    basis = gram_topr_basis(flat, r)
    codes = flat @ basis
    return codes.to(delta.dtype), basis.to(delta.dtype)


_chain_streams: dict[str, list] = {}
MAX_CHAIN_STREAMS = 8
USE_GRAPHS = True  # replay analytic_patches' layers as CUDA graphs after the first call


def _streams_for(device: torch.device, n: int) -> list:
    key = str(device)
    have = _chain_streams.setdefault(key, [])
    while len(have) < min(n, MAX_CHAIN_STREAMS):
        have.append(torch.cuda.Stream(device))
    return have


_PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def _layer_body(model, delta, l: int, x_in: Tensor, x_mid: Tensor, dx: Tensor, prop_r: int):
    """One layer of the engine loop from its stored inputs and the chain's ΔX: the dense ΔK / ΔV
    patch, the propagated ΔX before truncation, and the issued truncation job."""
    from deltakv_b200.subspace import gram_topr_begin

    cfg = model.cfg
    block = model.blocks[l]
    layer = delta.layers.get(l)
    xn, dxn = rmsnorm_first_order(x_in, dx, block.attn_norm.weight, cfg.rms_eps)
    dh, dk, dv, _ = attention_first_order(
        xn, dxn, block.q_proj.weight, block.k_proj.weight, block.v_proj.weight, block.o_proj.weight,
        layer, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, rope=model.rope)
    d1 = dx + dh
    xm, dxm = rmsnorm_first_order(x_mid, d1, block.mlp_norm.weight, cfg.rms_eps)
    d2 = (d1 + mlp_first_order(xm, dxm, block.gate_proj.weight, block.up_proj.weight, block.down_proj.weight,
                               layer)).float()
    # rank_truncate(d2, prop_r): codes = d2 @ basis, dX = codes @ basis^T
    return dk, dv, d2, gram_topr_begin(d2, prop_r)


def _signature(model, delta) -> tuple[list, tuple]:
    """Every tensor and scalar a captured layer bakes in: the tensors (checked by identity and
    version on each call) and the scalars (LoRA scales, shapes, eps, RoPE tables)."""
    cfg = model.cfg
    tensors, scalars = [], [float(cfg.rms_eps), int(cfg.n_heads), int(cfg.n_kv_heads), int(cfg.head_dim),
                            int(cfg.d_model), id(model.rope)]
    for l, block in enumerate(model.blocks):
        for name in ("attn_norm", "mlp_norm") + _PROJ:
            tensors.append(getattr(block, name).weight)
        layer = delta.layers.get(l)
        for name in _PROJ:
            fac = layer.get(name) if layer is not None else None
            if fac is not None:
                tensors += [fac.A, fac.B]
                scalars.append((l, name, float(getattr(fac, "scale", 1.0))))
    return tensors, tuple(scalars)


class _LayerGraphs:
    """CUDA graphs of every layer of analytic_patches for one (model, delta, shape)."""

    def __init__(self, model, delta):
        tensors, self.scalars = _signature(model, delta)
        self.refs = [weakref.ref(t) for t in tensors]
        self.versions = [t._version for t in tensors]
        self.layers: dict[int, dict] = {}
        self.keep: list = []

    def valid(self, model, delta) -> bool:
        tensors, scalars = _signature(model, delta)
        return (scalars == self.scalars and len(tensors) == len(self.refs)
                and all(r() is t and t._version == v for r, t, v in zip(self.refs, tensors, self.versions)))


_graph_sets: dict[tuple, object] = {}  # key -> _LayerGraphs, or False (not capturable); in LRU order
_graph_seen: dict[tuple, int] = {}    # eager calls per key (capture from the second one on)
MAX_GRAPH_SETS = 2                    # a set holds every layer's intermediates (GBs at 2k tokens)


def _capture(model, delta, hidden, chains, streams, prop_r, dev) -> _LayerGraphs | None:
    """Capture one graph per layer (each chain's layers in order on its stream): the layer's
    inputs are static buffers, step 0 starts from ΔX = 0 and step t > 0 from the previous
    layer's static ΔX and decided basis (``codes @ basis^T``)."""
    from deltakv_b200.subspace import _start_block

    gs = _LayerGraphs(model, delta)
    seq, d = int(hidden.seq_len), int(model.cfg.d_model)
    for c, chain in enumerate(chains):
        s = streams[c % len(streams)]
        prev = None
        for t, l in enumerate(chain):
            rec = {"x_in": torch.empty_like(hidden.layer_in(l), dtype=torch.float32),
                   "x_mid": torch.empty_like(hidden.layer_mid(l), dtype=torch.float32),
                   "basis": torch.zeros(d, prop_r, dtype=torch.float32, device=dev)}
            rec["x_in"].copy_(hidden.layer_in(l))
            rec["x_mid"].copy_(hidden.layer_mid(l))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                if prev is None:
                    dx = torch.zeros(seq, d, dtype=torch.float32, device=dev)
                else:
                    dx = (prev["d2"] @ prev["basis"]) @ prev["basis"].t()
                dk, dv, d2, job = _layer_body(model, delta, l, rec["x_in"], rec["x_mid"], dx, prop_r)
            if job.kind not in ("iter", "eig"):
                return None
            if job.kind == "iter":
                gs.keep.append(_start_block(1, d, job.k, dev))
            rec.update(graph=g, dk=dk, dv=dv, d2=d2, job=job, v=job.v, flags=job.flags)
            gs.layers[l] = rec
            prev = rec
    torch.cuda.synchronize(dev)
    return gs


def analytic_patches(hidden, delta, model, config) -> dict[int, LowRankKVPatch]:
    """The engine's analytic route (engine.py:377-432): per layer RMSNorm, first-order
    attention (the dense ΔK / ΔV patch), the residual update, first-order SwiGLU on the
    stored post-attention residual, and the rank-``propagator_rank`` truncation of ΔX;
    ΔX restarts from zero every ``hidden_stride`` layers.

    The layers between two restarts form a chain that depends on no other chain, so the
    chains run concurrently, each on its own stream (up to eight), with the same operations in
    the same order as one layer after another.  The host polls the chains' truncations
    (:func:`deltakv_b200.subspace.gram_topr_begin`, whose acceptance test is read on the host)
    and issues a chain's next layer as soon as its truncation is decided, while the other
    chains' kernels run.  From the third call with the same model, delta and shape on, each
    layer is one CUDA graph replay (captured after the second call; re-captured when a weight,
    factor or scale changes; at most MAX_GRAPH_SETS shapes keep their graphs), so the host
    issues a handful of operations per layer."""
    from deltakv_b200.subspace import gram_topr_finish

    cfg = model.cfg
    seq = int(hidden.seq_len)
    x0 = hidden.layer_in(0)
    ops._require_cuda(x0)
    dev = x0.device
    patches: dict[int, LowRankKVPatch] = {}
    n_layers = len(model.blocks)
    stride = max(1, int(config.hidden_stride))
    prop_r = max(1, min(int(config.propagator_rank), cfg.d_model, seq))
    chains = [range(s0, min(s0 + stride, n_layers)) for s0 in range(0, n_layers, stride)]
    cur = torch.cuda.current_stream(dev)
    half_tables(model.rope, dev)  # fill the per-device RoPE table cache on this stream before forking
    ops.status_word(dev)
    streams = _streams_for(dev, len(chains))  # side streams (a graph cannot be captured on the default one)
    fork = torch.cuda.Event()
    fork.record(cur)
    key = (id(model), id(delta), seq, str(dev), stride, prop_r, n_layers, id(streams[0]))
    gs = _graph_sets.get(key) if USE_GRAPHS else None
    if gs is not None and not (gs and gs.valid(model, delta)):
        if gs:  # stale: a weight, factor or scale changed
            _graph_sets.pop(key, None)
        gs = None
    if gs:
        _graph_sets[key] = _graph_sets.pop(key)  # most recently used last
    dx: list[Tensor | None] = [None] * len(chains)

    def issue(c: int, step: int):
        l = chains[c][step]
        s = streams[c % len(streams)]
        with torch.cuda.stream(s):
            if step == 0 and s != cur:
                s.wait_event(fork)
            if gs is not None:
                rec = gs.layers[l]
                rec["x_in"].copy_(hidden.layer_in(l))
                rec["x_mid"].copy_(hidden.layer_mid(l))
                rec["graph"].replay()
                job = rec["job"]
                job.v, job.flags, job.stream = rec["v"], rec["flags"], s
                job.done = torch.cuda.Event()
                job.done.record(s)
                return job, rec, s, step
            if step == 0:
                dx[c] = torch.zeros(seq, cfg.d_model, dtype=torch.float32, device=dev)
            dk, dv, d2, job = _layer_body(model, delta, l, hidden.layer_in(l), hidden.layer_mid(l), dx[c], prop_r)
            return job, {"dk": dk, "dv": dv, "d2": d2}, s, step

    pending = {c: issue(c, 0) for c in range(len(chains))}
    while pending:
        ready = [c for c, (job, _, _, _) in pending.items() if job.ready()]
        if not ready:
            time.sleep(2e-5)
            continue
        for c in ready:
            job, rec, s, step = pending.pop(c)
            l = chains[c][step]
            with torch.cuda.stream(s):
                basis = gram_topr_finish([job])[0]
                if gs is not None:
                    rec["basis"].copy_(basis)  # read by the next layer's graph
                    dk, dv = rec["dk"].clone(), rec["dv"].clone()
                else:
                    dx[c] = (rec["d2"] @ basis) @ basis.t()
                    dk, dv = rec["dk"], rec["dv"]
            patches[l] = LowRankKVPatch(layer_idx=l, k_codes=None, k_basis=None, v_codes=None, v_basis=None,
                                        k_dense=dk, v_dense=dv)
            if step + 1 < len(chains[c]):
                pending[c] = issue(c, step + 1)
    if any(s != cur for s in streams):
        for s in streams:
            if s != cur:
                e = torch.cuda.Event()
                e.record(s)
                cur.wait_event(e)
        for p in patches.values():  # made on the chain streams, used on the caller's
            p.k_dense.record_stream(cur)
            p.v_dense.record_stream(cur)
    if USE_GRAPHS and key not in _graph_sets:
        # a shape seen once is not captured (one-off lengths would each cost a capture and a
        # set of graph memory); from the second eager call on it is, evicting the least
        # recently used set beyond MAX_GRAPH_SETS
        _graph_seen[key] = _graph_seen.get(key, 0) + 1
        if _graph_seen[key] >= 2:
            live = [k for k, v in _graph_sets.items() if v]
            while len(live) >= MAX_GRAPH_SETS:
                _graph_sets.pop(live.pop(0), None)
            try:
                _graph_sets[key] = _capture(model, delta, hidden, chains, streams, prop_r, dev) or False
            except RuntimeError:
                _graph_sets[key] = False  # not capturable here: stay on the eager path
            _graph_seen.pop(key, None)
    return patches
