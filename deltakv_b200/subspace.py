"""Subspace route on the B200 kernels.

Drop-in for ``deltakv.patches.subspace.subspace_correct`` (src/deltakv/patches/subspace.py:45-106)
and ``svd_basis`` (37-42).  The per-token work (residual, least-squares codes onto col(B),
fitted field, CacheBlend-style weights, probe override) runs in ``libdkv_b200.so``; the K
path's basis — the top right singular subspace of the gathered [n_probes, d] probe residual —
comes from :func:`topr_basis` (block subspace iteration with a device Rayleigh-Ritz step, the
exact SVD where its convergence estimate is not met); :func:`svd_basis` is the library SVD.
"""

from __future__ import annotations

import ctypes as C
import math
import weakref

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


def _orthonormalize(z: Tensor) -> tuple[Tensor, Tensor]:
    """Orthonormal basis of the columns of ``z [b, d, k]``: Cholesky QR applied twice in fp64
    (CholQR2: Fukaya, Nakatsukasa et al., 2014).  Returns the basis and a device flag per batch
    element whose Gram matrix was not numerically positive definite (its basis is then
    meaningless and the caller recomputes it) — no host synchronisation."""
    q = z.double()
    bad = torch.zeros(q.shape[0], dtype=torch.bool, device=q.device)
    for _ in range(2):
        g = torch.matmul(q.transpose(1, 2), q)
        l, info = torch.linalg.cholesky_ex(g)
        bad |= info != 0
        q = torch.linalg.solve_triangular(l, q.transpose(1, 2), upper=False).transpose(1, 2)
    return q.float(), bad


def sym_eig(t: Tensor, *, max_sweeps: int = 30) -> tuple[Tensor, Tensor, Tensor]:
    """Eigendecomposition of the symmetric ``t [b, k, k]`` (k <= 96) on the device, fp64:
    ``(evals [b, k] descending, evecs [b, k, k] with column j for evals[:, j], info [b])``,
    info 0 converged, 1 not converged in ``max_sweeps`` Jacobi sweeps, 2 non-finite input."""
    ops._require_cuda(t)
    a = t.to(torch.float64).contiguous()
    b, k = int(a.shape[0]), int(a.shape[-1])
    ev = torch.empty(b, k, dtype=torch.float64, device=a.device)
    vec = torch.empty(b, k, k, dtype=torch.float64, device=a.device)
    info = torch.empty(b, dtype=torch.int32, device=a.device)
    rc = L.lib().dkv_sym_eig_batched(a.data_ptr(), b, k, k * k, int(max_sweeps), ev.data_ptr(), vec.data_ptr(),
                                     info.data_ptr(), ops.stream_ptr())
    L.check(rc, "dkv_sym_eig_batched")
    return ev, vec, info


MAX_RITZ = 96  # largest rank + oversample the device eigensolver takes
_start_cache: dict[tuple, tuple[Tensor, Tensor]] = {}


def _start_block(n_b: int, d: int, k: int, device: torch.device) -> tuple[Tensor, Tensor]:
    key = (str(device), n_b, d, k)
    hit = _start_cache.get(key)
    if hit is None:
        if len(_start_cache) >= 8:
            _start_cache.clear()
        gen = torch.Generator(device=device).manual_seed(1234)
        hit = _orthonormalize(torch.randn(n_b, d, k, generator=gen, device=device))
        torch.cuda.current_stream(device).synchronize()  # once per shape: usable from any stream
        _start_cache[key] = hit
    cur = torch.cuda.current_stream(device)
    if not torch.cuda.is_current_stream_capturing():  # a graph holds its own reference instead
        for t in hit:
            t.record_stream(cur)  # kept from reuse until this stream's work is done, if evicted
    return hit


THIN_MAX_N = 96  # widest product the split-precision thin GEMM takes


def thin_mm(a: Tensor, b: Tensor, *, trans_a: bool = False) -> Tensor:
    """``op(a) @ b`` for fp32 ``a [bt, m, k]`` (``trans_a``: ``a [bt, k, m]``, used transposed)
    and ``b [bt, k, n]``: the subspace iteration's thin products on the tensor cores with
    split-precision operands (``dkv_split_gemm_batched``, within ~1e-5 relative of fp32).  The
    result is ``[bt, m, n16]`` with ``n16`` = n rounded up to 16 (columns past n are zero, so it
    can be passed on as the next product's ``b`` as it is); shapes the kernel does not take go to
    the library GEMM and come back ``[bt, m, n]``."""
    bt = int(a.shape[0])
    m, k = (int(a.shape[2]), int(a.shape[1])) if trans_a else (int(a.shape[1]), int(a.shape[2]))
    n = int(b.shape[2])
    n16 = (n + 15) // 16 * 16
    ok = (a.is_cuda and a.dtype == torch.float32 and b.dtype == torch.float32 and 0 < n16 <= THIN_MAX_N
          and bt <= 65535 and a.stride(2) == 1 and a.stride(1) % 4 == 0 and a.stride(0) % 4 == 0
          and a.data_ptr() % 16 == 0 and (m % 4 == 0 if trans_a else k % 4 == 0))
    if not ok:
        return torch.matmul(a.transpose(1, 2) if trans_a else a, b)
    if (b.shape[2] != n16 or b.stride(2) != 1 or b.stride(1) % 4 or b.stride(0) % 4 or b.data_ptr() % 16):
        bp = torch.zeros(bt, k, n16, dtype=torch.float32, device=b.device)
        bp[:, :, :n] = b
        b = bp
    out = torch.empty(bt, m, n16, dtype=torch.float32, device=a.device)
    rc = L.lib().dkv_split_gemm_batched(a.data_ptr(), a.stride(0), a.stride(1), int(trans_a), b.data_ptr(),
                                        b.stride(0), b.stride(1), out.data_ptr(), out.stride(0), out.stride(1), bt,
                                        m, n16, k, ops.stream_ptr())
    L.check(rc, "dkv_split_gemm_batched")
    return out


def _ritz(x: Tensor, q: Tensor, r: int) -> tuple[Tensor, Tensor, Tensor]:
    """Rayleigh-Ritz on span(q): the top-``r`` Ritz vectors of ``x^T x`` and all Ritz values."""
    w = thin_mm(x, q)[:, :, :q.shape[2]]
    ev, vec, info = sym_eig(torch.matmul(w.transpose(1, 2), w))
    return torch.matmul(q, vec[:, :, :r].float()), ev, info


def gram_basis(x: Tensor, rank: int) -> Tensor:
    """Leading-``rank`` right singular subspace of ``x [..., m, d]`` as ``[..., d, rank]`` from
    the eigenvectors of the fp64 Gram matrix ``x^T x`` (a library eigensolver, batched): the
    exact path of :func:`topr_basis`, more accurate than an fp32 SVD (the Gram matrix of fp32
    data is formed to ~1e-16 in fp64) and several times faster for d up to a few thousand."""
    xd = x.double()
    c = torch.matmul(xd.transpose(-1, -2), xd)
    _, v = torch.linalg.eigh(c)  # ascending eigenvalues
    return v[..., :, -rank:].flip(-1).to(x.dtype).contiguous()


GRAM_TOL = 1e-6  # estimated ||x (P - P_exact)||_F / ||x||_F accepted from the iteration
gram_launches = 0  # kernels of this library launched by gram_topr_basis so far (a running count)


def _eigh_top(c: Tensor, rank: int) -> Tensor:
    _, v = torch.linalg.eigh(c)  # ascending eigenvalues
    return v[:, -rank:].flip(-1)


class GramJob:
    """One :func:`gram_topr_begin` computation in flight on the stream it was issued on."""

    __slots__ = ("x_dtype", "r", "k", "d", "c", "q", "y", "w", "t", "st", "trace", "v", "flags", "stream",
                 "done", "kind", "iters")

    def ready(self) -> bool:
        """Whether :func:`gram_topr_finish` would find this job's flags computed (no wait)."""
        return self.done is None or self.done.query()


def _gram_run(job: GramJob, n_it: int) -> None:
    """``n_it`` more iteration steps from ``job.q``, the Rayleigh-Ritz step, and the device
    flags ``[estimate, rate, eigensolver info, breakdown status]`` — no synchronisation."""
    global gram_launches
    gram_launches += 2 * int(n_it) + 2  # n_it x (G Q, Cholesky QR), the Rayleigh quotient, Jacobi
    c, q, r, k = job.c, job.q, job.r, job.k
    rc = L.lib().dkv_gram_subspace_iterate(c.data_ptr(), job.d, q.data_ptr(), k, int(n_it), job.y.data_ptr(),
                                           job.w.data_ptr(), job.t.data_ptr(), job.st.data_ptr(), ops.stream_ptr())
    L.check(rc, "dkv_gram_subspace_iterate")
    ev, vec, info = sym_eig(job.t[None])
    ev, vec = ev[0], vec[0]
    v = torch.matmul(q, vec[:, :r])
    res = torch.matmul(c, v) - v * ev[:r]
    est = res.norm() / (ev[r - 1] - ev[r]) * torch.sqrt(ev[r - 1].clamp_min(0.0) / job.trace)
    rate = ev[k - 1] / ev[r - 1]
    job.v = v
    job.flags = torch.stack([est, rate, info[0].double(), job.st[0].double()])
    job.done = None
    if not torch.cuda.is_current_stream_capturing():  # a replayed graph's caller records it
        job.done = torch.cuda.Event()
        job.done.record(job.stream)


def gram_topr_begin(x: Tensor, rank: int, *, oversample: int = 32, iters: int = 28) -> GramJob:
    """Issue :func:`gram_topr_basis` for ``x [m, d]`` on the current stream without a host
    synchronisation; :func:`gram_topr_finish` completes any number of such jobs with one."""
    ops._require_cuda(x)
    global gram_launches
    job = GramJob()
    m, d = int(x.shape[0]), int(x.shape[1])
    job.x_dtype, job.d, job.r = x.dtype, d, max(1, min(int(rank), m, d))
    job.stream = torch.cuda.current_stream(x.device)
    job.iters = int(iters)
    job.flags = job.done = job.v = None
    xd = x.double()
    job.c = torch.matmul(xd.transpose(0, 1), xd)
    job.k = min(job.r + oversample, MAX_RITZ)
    if d <= MAX_RITZ:
        job.kind = "eig"
        ev, vec, info = sym_eig(job.c[None])
        gram_launches += 1
        job.v = vec[0, :, :job.r]
        job.flags = info[0].double()[None]
        if not torch.cuda.is_current_stream_capturing():
            job.done = torch.cuda.Event()
            job.done.record(job.stream)
        return job
    if job.k - job.r < 8 or m < job.k:  # too little oversampling, or a Gram matrix of rank < k
        job.kind = "exact"
        return job
    job.kind = "iter"
    dev = x.device
    job.q = _start_block(1, d, job.k, dev)[0][0].double().contiguous()
    job.y = torch.empty(d, job.k, dtype=torch.float64, device=dev)
    job.w = torch.empty(2, job.k, job.k, dtype=torch.float64, device=dev)
    job.t = torch.empty(job.k, job.k, dtype=torch.float64, device=dev)
    job.st = torch.empty(1, dtype=torch.int32, device=dev)
    job.trace = job.c.diagonal().sum()
    _gram_run(job, job.iters)
    return job


def gram_topr_finish(jobs: list[GramJob], *, tol: float | None = None) -> list[Tensor]:
    """The bases of ``jobs`` (each ``[d, rank]``, in its job's dtype, produced on its job's
    stream): one host synchronisation reads every job's flags; a job whose estimate misses
    ``tol`` (default :data:`GRAM_TOL`) continues or takes the exact path on its own stream."""
    if not jobs:
        return []
    tol = GRAM_TOL if tol is None else float(tol)
    cur = torch.cuda.current_stream(jobs[0].c.device)
    live = [j for j in jobs if j.flags is not None]
    host: list[list[float]] = []
    if live:
        for j in live:
            if j.stream != cur:
                cur.wait_event(j.done)
        flat = torch.cat([j.flags for j in live]).cpu().tolist()
        pos = 0
        for j in live:
            host.append(flat[pos:pos + j.flags.numel()])
            pos += j.flags.numel()
    out, it = [], iter(host)
    for j in jobs:
        f = next(it) if j.flags is not None else None
        with torch.cuda.stream(j.stream):
            out.append(_gram_decide(j, f, tol).to(j.x_dtype).contiguous())
    return out


def _gram_decide(job: GramJob, f, tol: float) -> Tensor:
    if job.kind == "eig":
        return job.v if f[0] == 0 else _eigh_top(job.c, job.r)
    if job.kind == "exact":
        return _eigh_top(job.c, job.r)
    est, rate, good = f[0], f[1], f[2] == 0 and f[3] == 0 and f[0] == f[0]  # converged, no breakdown, not NaN
    if good and 0.0 <= est <= tol:
        return job.v
    if good and est < float("inf") and 0.0 < rate < 1.0:
        more = int(math.ceil(math.log(est / tol) / -math.log(rate))) + 2
        if more <= 2 * job.iters:
            _gram_run(job, more)
            g = job.flags.cpu().tolist()
            if g[2] == 0 and g[3] == 0 and g[0] == g[0] and 0.0 <= g[0] <= tol:
                return job.v
    return _eigh_top(job.c, job.r)


def gram_topr_basis(x: Tensor, rank: int, *, oversample: int = 32, iters: int = 28,
                    tol: float | None = None) -> Tensor:
    """Leading-``rank`` right singular subspace of ``x [m, d]`` as ``[d, rank]`` (Ritz vectors
    of ``x^T x``, descending) for spectra without a gap at ``rank`` — the analytic route's
    propagated dX, whose singular values at the cut differ by ~1 % (rank_truncate,
    src/deltakv/patches/analytic.py:14-22).

    The fp64 Gram matrix ``C = x^T x`` is formed once; ``iters`` steps of block subspace
    iteration with ``k = rank + oversample`` columns (at most 96) and Cholesky QR run on it in
    two fused kernels per step (``dkv_gram_subspace_iterate``), then one Rayleigh-Ritz step on
    the device Jacobi eigensolver (Golub & Van Loan, Matrix Computations 4th ed., Sec. 8.2.4).
    The subspace error shrinks by ``l_k / l_rank`` per step however close ``l_rank`` and
    ``l_rank+1`` are: the Ritz step resolves them exactly within span(Q).  Accepted when
    ``||C V - V Theta||_F / (theta_r - theta_r+1) * sqrt(theta_r / tr C)`` — the residual bound on
    the subspace angle (Davis-Kahan) weighted by the singular value at the cut, an estimate of
    ``||x (P - P_exact)||_F / ||x||_F`` that measured 10-20x above the true error on such data —
    is at most ``tol``; otherwise the iteration continues once by the number of steps the Ritz
    values' rate predicts, and failing that (or on a Cholesky breakdown) the exact path (library
    eigensolver on C) is used.  One host synchronisation per decision.  ``d <= 96``: the device
    eigensolver on C directly."""
    return gram_topr_finish([gram_topr_begin(x, rank, oversample=oversample, iters=iters)], tol=tol)[0]


def topr_basis(residual: Tensor, rank: int, *, iters: int = 3, min_iters: int = 2, oversample: int = 8) -> Tensor:
    """Leading-``rank`` right singular subspace of ``residual [..., m, d]`` as ``[..., d, rank]``,
    batched over a leading dimension.

    The same subspace as :func:`svd_basis` (the reference's ``svd_basis``,
    src/deltakv/patches/subspace.py:37-42), computed by block subspace iteration on
    ``C = R^T R`` — applied as ``R^T (R Q)``, never formed — with re-orthonormalisation and a
    Rayleigh-Ritz step (Golub & Van Loan, Matrix Computations, 4th ed., Sec. 8.2.4; Halko,
    Martinsson & Tropp, SIAM Review 2011, Alg. 4.4) on ``k = rank + oversample`` columns
    instead of a full SVD; the thin products run on the tensor cores with split-precision
    operands (:func:`thin_mm`) and the k x k Rayleigh-Ritz eigenproblem on the device
    (:func:`sym_eig`).  The subspace converges as ``(l_k / l_rank)^i`` after ``i`` products
    (eigenvalues of C); the least-squares correction depends on the basis only through its
    column space, so the rotation within the subspace is immaterial.  Every element gets
    ``min_iters`` iterations; those whose Ritz values then estimate a subspace error above
    ``1e-5`` continue to ``iters`` when that estimate, extrapolated, could still get there;
    the rest — and any whose orthonormalisation or eigensolve failed — take the exact path
    (:func:`gram_basis`), so the result never depends on a half-converged iteration.  One host
    synchronisation per decision.
    """
    ops._require_cuda(residual)
    x = residual.float()
    batched = x.ndim == 3
    if not batched:
        x = x.unsqueeze(0)
    n_b, m, d = x.shape
    r = max(1, min(int(rank), m, d))
    k = min(d, r + oversample)
    if k >= m or k > MAX_RITZ:
        basis = gram_basis(x, r)
        return basis if batched else basis[0]
    first = max(1, min(int(min_iters), int(iters)))
    tol = 1e-5

    def iterate(xb: Tensor, q: Tensor, bad: Tensor, n: int) -> tuple[Tensor, Tensor]:
        for _ in range(n):
            z = thin_mm(xb, thin_mm(xb, q), trans_a=True)[:, :, :q.shape[2]]  # X^T (X Q)
            q, b2 = _orthonormalize(z)
            bad = bad | b2
        return q, bad

    def estimate(ev: Tensor, done: int) -> Tensor:
        if k >= d:
            return torch.zeros_like(ev[:, 0])
        return (ev[:, k - 1].clamp_min(0.0) / ev[:, r - 1].clamp_min(1e-300)) ** done

    def failed(info: Tensor, bad: Tensor, est: Tensor) -> Tensor:
        return bad | (info != 0) | ~torch.isfinite(est)

    q0, bad0 = _start_block(n_b, d, k, x.device)
    q, bad = iterate(x, q0, bad0, first)
    basis, ev, info = _ritz(x, q, r)
    est = estimate(ev, first)
    more = int(iters) - first
    # continue only where the extrapolated estimate after all iterations meets the tolerance
    hopeless = failed(info, bad, est) | (est ** (float(iters) / first) > tol)
    settled = ~hopeless & (est <= tol)
    flags = torch.stack([settled, hopeless]).cpu()  # the host decision
    cont = torch.nonzero(~flags[0] & ~flags[1]).view(-1).to(x.device) if more > 0 else None
    exact = [torch.nonzero(flags[1]).view(-1)]
    if more <= 0:
        exact.append(torch.nonzero(~flags[0] & ~flags[1]).view(-1))
    elif cont.numel():
        xs = x[cont]
        qs, bads = iterate(xs, q[cont], bad[cont], more)
        bsub, evs, infos = _ritz(xs, qs, r)
        basis[cont] = bsub
        e2 = estimate(evs, int(iters))
        exact.append(cont[(failed(infos, bads, e2) | (e2 > tol)).nonzero().view(-1)].cpu())
    redo = torch.cat(exact).to(x.device)
    if redo.numel():
        basis[redo] = gram_basis(x[redo], r)
    return basis if batched else basis[0]


def _rows(t: Tensor) -> Tensor:
    r = t.reshape(t.shape[0], -1)
    if r.stride(1) != 1:
        r = r.contiguous()
    return r


_rows_seen: dict[int, tuple] = {}  # id(probe tensor) -> (weakref, version, seq, device, rows)


def _probe_rows(probe_index: Tensor, seq: int, dev: torch.device) -> Tensor:
    """The probe index as int32 rows in [0, seq) (negative entries count from the end, as torch
    indexing does); out-of-range entries raise the reference's IndexError.  The check reads
    the index on the host; its result is kept for as long as the same tensor lives unmodified
    (its in-place version counter), so a caller that passes one probe set to many calls pays
    the host round trip once."""
    key = id(probe_index)
    hit = _rows_seen.get(key)
    if (hit is not None and hit[0]() is probe_index and hit[1] == probe_index._version and hit[2] == seq
            and hit[3] == str(dev)):
        return hit[4]
    rows = _check_probe_rows(probe_index, seq, dev)
    if len(_rows_seen) >= 64:
        _rows_seen.clear()
    try:
        _rows_seen[key] = (weakref.ref(probe_index), probe_index._version, seq, str(dev), rows)
    except TypeError:  # not weak-referenceable: no caching
        pass
    return rows


def _check_probe_rows(probe_index: Tensor, seq: int, dev: torch.device) -> Tensor:
    idx = probe_index.to(device=dev, dtype=torch.int64).reshape(-1)
    if idx.numel():
        lo, hi = int(idx.min()), int(idx.max())
        if lo < -seq or hi >= seq:
            bad = hi if hi >= seq else lo
            raise IndexError(f"index {bad} is out of bounds for dimension 0 with size {seq}")
        idx = torch.where(idx < 0, idx + seq, idx)
    return idx.to(torch.int32).contiguous()


def _prepare(reused: Tensor, fresh: Tensor, probe_index: Tensor, basis: Tensor | None, rank: int,
             token_weights: Tensor | None, rows_cache: dict | None = None, sub_mu: tuple | None = None):
    """Checks and device views of one problem: ``(args without workspace, tensors to keep alive,
    (corrected, subspace, orth_mu, shape, result dtype))``.  ``rows_cache`` shares one probe
    index's checked rows between the problems of a batch (one host round trip, not one each);
    ``sub_mu`` gives zeroed fp32 ``[d]`` outputs for subspace and orth_mu (views of a batch's
    arrays) instead of two fresh ones."""
    ops._require_cuda(reused, fresh)
    seq, n_kv, hd = reused.shape
    dev = reused.device
    key = (probe_index.data_ptr(), probe_index.numel(), probe_index.dtype, seq, str(dev))
    idx = None if rows_cache is None else rows_cache.get(key)
    if idx is None:
        idx = _probe_rows(probe_index, seq, dev)
        if rows_cache is not None:
            rows_cache[key] = idx
    rf, ff = _rows(reused), _rows(fresh)
    if ff.dtype != rf.dtype:
        ff = ff.to(rf.dtype)
    d = rf.shape[1]
    if basis is None:
        r_eff = min(rank, max(1, int(idx.numel()) - 1), d)
        basis = topr_basis(probe_residual(rf, ff, idx), r_eff) if idx.numel() >= 2 else None
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
    if sub_mu is None:
        sub = torch.zeros(d, dtype=torch.float32, device=dev)
        mu = torch.zeros(d, dtype=torch.float32, device=dev)
    else:
        sub, mu = sub_mu
    tw = None
    if token_weights is not None:
        tw = token_weights.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    args = L.SubspaceArgs(
        reused=rf.data_ptr(), fresh=ff.data_ptr(), kv_dtype=ops.dkv_dtype(rf.dtype), n_tokens=seq, d=d,
        reused_row_stride=rf.stride(0), fresh_row_stride=ff.stride(0),
        probe_index=idx.data_ptr() if idx.numel() else None, n_probes=idx.numel(),
        basis=ops.ptr(b32), rank=r, token_weights=ops.ptr(tw),
        corrected=corr.data_ptr(), out_dtype=ops.dkv_dtype(out_dtype), out_row_stride=corr.stride(0),
        subspace_out=sub.data_ptr(), orth_mu_out=mu.data_ptr(), workspace=None, workspace_bytes=0,
    )
    return args, (rf, ff, idx, b32, tw), (corr, sub, mu, (seq, n_kv, hd), reused.dtype)


def _finish(out):
    corr, sub, mu, (seq, n_kv, hd), res_dtype = out
    return corr.view(seq, n_kv, hd).to(res_dtype), sub.to(res_dtype), mu.to(res_dtype)


def _run_one(args, dev) -> None:
    nbytes = workspace_bytes(args.n_tokens, args.d, args.rank)
    ws = _workspace(dev, nbytes)
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    L.check(L.lib().dkv_subspace_correct(C.byref(args), ops.stream_ptr()), "dkv_subspace_correct")


def subspace_correct(reused: Tensor, fresh: Tensor, probe_index: Tensor, *, basis: Tensor | None = None,
                     rank: int = 8, token_weights: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """Correct ``reused`` toward ``fresh`` in a rank-r subspace plus an orthogonal shift.

    Returns ``(corrected [seq, n_kv, hd], subspace_offset [d], orth_mu [d])`` like the reference.
    """
    args, keep, out = _prepare(reused, fresh, probe_index, basis, rank, token_weights)
    _run_one(args, reused.device)
    return _finish(out)


MAX_BATCH = 112  # problems per batched launch set


def subspace_correct_batched(problems: list[dict]) -> list[tuple[Tensor, Tensor, Tensor]]:
    """:func:`subspace_correct` for many problems (keyword dicts of its arguments: ``reused``,
    ``fresh``, ``probe_index``, optional ``basis``, ``rank``, ``token_weights``) in one set of
    launches (``dkv_subspace_correct_batched``) — the per-layer K / V loop of the reference's
    apply_probe_to_cache (src/deltakv/patches/probe.py:112-165).  Problems the batched form
    does not take (d not a multiple of 32, unaligned rows, mixed d or dtype) run one by one."""
    if not problems:
        return []
    rows_cache: dict = {}
    # one zeroed [count, d] array per (d, device) for every problem's subspace and orth_mu
    # outputs, instead of two small allocations (and fills) per problem
    groups: dict = {}
    for i, p in enumerate(problems):
        r = p["reused"]
        groups.setdefault((r.shape[-2] * r.shape[-1], str(r.device)), []).append(i)
    sub_mu = [None] * len(problems)
    blocks = []
    for (d, _), ids in groups.items():
        dev_ = problems[ids[0]]["reused"].device
        sm = torch.zeros(2, len(ids), d, dtype=torch.float32, device=dev_)
        blocks.append((ids, sm))
        for j, i in enumerate(ids):
            sub_mu[i] = (sm[0, j], sm[1, j])
    preps = [_prepare(p["reused"], p["fresh"], p["probe_index"], p.get("basis"), p.get("rank", 8),
                      p.get("token_weights"), rows_cache, sub_mu[i]) for i, p in enumerate(problems)]
    dev = problems[0]["reused"].device
    for lo in range(0, len(preps), MAX_BATCH):
        chunk = preps[lo:lo + MAX_BATCH]
        arr = (L.SubspaceArgs * len(chunk))(*[a for a, _, _ in chunk])
        nbytes = C.c_int64()
        rc = L.lib().dkv_subspace_correct_batched_workspace_bytes(arr, len(chunk), C.byref(nbytes))
        if rc == L.DKV_ERR_UNSUPPORTED:
            for a, _, _ in chunk:
                _run_one(a, dev)
            continue
        L.check(rc, "dkv_subspace_correct_batched_workspace_bytes")
        ws = _workspace(dev, nbytes.value)
        L.check(L.lib().dkv_subspace_correct_batched(arr, len(chunk), ws.data_ptr(), ws.numel(), ops.stream_ptr()),
                "dkv_subspace_correct_batched")
    # subspace and orth_mu in each problem's dtype: one conversion per block and dtype
    conv: dict = {}
    for ids, sm in blocks:
        for dt in {problems[i]["reused"].dtype for i in ids}:
            conv[(id(sm), dt)] = sm if dt == torch.float32 else sm.to(dt)
    results = [None] * len(problems)
    for ids, sm in blocks:
        for j, i in enumerate(ids):
            corr, _, _, (seq, n_kv, hd), res_dtype = preps[i][2]
            c = conv[(id(sm), res_dtype)]
            results[i] = (corr.view(seq, n_kv, hd).to(res_dtype), c[0, j], c[1, j])
    return results
