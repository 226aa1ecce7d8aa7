"""Batched subspace correction of KIVI int4 caches on the GPU vs the oracle composition
(oracle KIVI dequantise -> oracle subspace_correct (fp32, the reference's precision) -> oracle
KIVI quantise).

The kernel carries its tensor-core operands as two bf16 terms each (products within ~2^-15
relative of fp32), so its corrected values differ from the oracle's fp32 ones by ~1e-5 of
the fitted part — about 1e-6 of an int4 step.  The int4 output therefore has to match the
oracle's bit for bit except where the oracle's own value sits that close to a rounding tie:

* fp16 scale and zero bits equal for every group, except groups whose fp32 scale
  (max - min) / 15 or zero (min) lies within 2e-5 relative of an fp16 rounding tie;
* in the groups whose scale and zero match, every int4 code equal, except codes whose
  oracle quotient (x - z) / s lies within 1e-3 of a rounding tie (and those differ by one);
* >= 99.9 % of all codes equal;
* orth_mu and subspace within 1e-5 relative (L2) of the oracle's plus 1e-5 of the mean
  residual norm (both are means of per-token quantities that largely cancel).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200 import kivi as K
from oracle import kivi as OK
from oracle import subspace as OS

pytestmark = pytest.mark.gpu


def _case(gen, n, n_kv, hd, r, mode, probe_ratio=0.1, drift=0.05):
    d = n_kv * hd
    base_f = torch.randn(n, d, generator=gen)
    B = torch.randn(d, max(r, 1), generator=gen) / d ** 0.5
    codes = torch.randn(n, max(r, 1), generator=gen) * 0.3
    fresh = base_f + codes @ B.T + drift * torch.randn(d, generator=gen) + 0.01 * torch.randn(n, d, generator=gen)
    n_p = max(0, int(round(probe_ratio * n)))
    probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.long), torch.randperm(n, generator=gen)[:n_p]]))
    c, s, z = OK.quantize(base_f.numpy(), mode)
    return dict(d=d, n_kv=n_kv, hd=hd, c=c, s=s, z=z, fresh=fresh, probes=probes, B=B[:, :r] if r else None, mode=mode)


def _oracle(cs):
    reused = OK.dequantize(cs["c"], cs["s"], cs["z"], cs["mode"])
    n = reused.shape[0]
    corr, sub, mu = OS.subspace_correct(reused.reshape(n, cs["n_kv"], cs["hd"]),
                                        cs["fresh"].numpy().reshape(n, cs["n_kv"], cs["hd"]),
                                        cs["probes"].numpy(), basis=None if cs["B"] is None else cs["B"].numpy(),
                                        rank=0 if cs["B"] is None else cs["B"].shape[1])
    corr = corr.reshape(n, -1)
    return corr, sub, mu, OK.quantize(corr, cs["mode"])


def _device_base(cs, dev):
    kt = K.KiviTensor(torch.from_numpy(cs["c"]).to(dev), torch.from_numpy(cs["s"]).to(dev),
                      torch.from_numpy(cs["z"]).to(dev), cs["mode"])
    return kt


def _near_f16_tie(x: np.ndarray, rel: float = 2e-5) -> np.ndarray:
    """Values whose float16 rounding changes within +-rel relative (a rounding tie nearby)."""
    x = np.asarray(x, np.float32)
    lo = (x * np.float32(1 - rel)).astype(np.float16)
    hi = (x * np.float32(1 + rel)).astype(np.float16)
    return lo != hi


def _groups(a: np.ndarray, mode: str, n: int) -> np.ndarray:
    """Per-element view of a per-group array: V [n, d/32] -> [n, d], K [ceil(n/32), d] -> [n, d]."""
    return np.repeat(a, 32, axis=1) if mode == "v" else np.repeat(a, 32, axis=0)[:n]


def _group_extrema(corr: np.ndarray, mode: str):
    n, d = corr.shape
    if mode == "v":
        g = corr.reshape(n, d // 32, 32)
        return g.min(-1), g.max(-1)
    ng = (n + 31) // 32
    lo = np.stack([corr[32 * i:32 * i + 32].min(0) for i in range(ng)])
    hi = np.stack([corr[32 * i:32 * i + 32].max(0) for i in range(ng)])
    return lo, hi


def _check(cs, out, sub, mu, tag, stats=None):
    corr, osub, omu, (oc, osc, oz) = _oracle(cs)
    mode = cs["mode"]
    got_c = out.codes.cpu().numpy()
    got_s = out.scale.cpu().numpy()
    got_z = out.zero.cpu().numpy()
    n, d = corr.shape
    # fp16 scale / zero: bit-equal unless the oracle's fp32 value is at an fp16 tie
    lo, hi = _group_extrema(corr, mode)
    s32 = (np.maximum(hi - lo, np.float32(1e-8)) / np.float32(15)).astype(np.float32)
    sz_eq = (got_s.view(np.uint16) == osc.view(np.uint16)) & (got_z.view(np.uint16) == oz.view(np.uint16))
    sz_tie = _near_f16_tie(s32) | _near_f16_tie(lo)
    assert (sz_eq | sz_tie).all(), (tag, int((~sz_eq & ~sz_tie).sum()))
    # codes: equal within groups whose parameters match, except next to a rounding tie
    gq, oq = OK.unpack_nibbles(got_c), OK.unpack_nibbles(oc)
    same = _groups(sz_eq, mode, n)
    s_el = _groups(osc.astype(np.float32), mode, n)
    z_el = _groups(oz.astype(np.float32), mode, n)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = (corr - z_el) / s_el
    tie = np.abs(y - np.floor(y) - 0.5) < 1e-3
    bad = same & (gq != oq) & ~(tie & (np.abs(gq.astype(int) - oq.astype(int)) == 1))
    assert not bad.any(), (tag, int(bad.sum()))
    eq_codes = float((gq == oq).mean())
    assert eq_codes >= 0.999, (tag, eq_codes)
    deq = OK.dequantize(got_c, got_s, got_z, mode)
    step = _groups(got_s.astype(np.float32), mode, n)
    span = float(np.abs(corr).max())
    assert (np.abs(deq - corr) <= 0.5 * step * 1.01 + 1e-5 * span).all(), tag
    errs = []
    if sub is not None and cs["B"] is not None and cs["probes"].numel() > 0:
        reused = OK.dequantize(cs["c"], cs["s"], cs["z"], mode)
        mean_dist = float(np.linalg.norm(cs["fresh"].numpy() - reused, axis=1).mean())
        for got, want in ((mu.cpu().numpy(), omu), (sub.cpu().numpy(), osub)):
            err = float(np.linalg.norm(got - want))
            errs.append(err / (np.linalg.norm(want) + mean_dist))
            assert err < 1e-5 * (np.linalg.norm(want) + mean_dist), (tag, err, float(np.linalg.norm(want)))
    print("kivi-subspace", tag, "codes equal", eq_codes, "scale/zero equal", float(sz_eq.mean()), "mu/sub", errs)
    if stats is not None:
        stats.append((tag, eq_codes, float(sz_eq.mean()), errs))


@pytest.mark.parametrize("mode", ["v", "k"])
@pytest.mark.parametrize("n,n_kv,hd,r,fdt,inplace", [
    (300, 2, 64, 8, torch.float32, False),
    (1000, 8, 128, 16, torch.bfloat16, True),
    (77, 4, 32, 64, torch.float32, False),
    (256, 1, 64, 48, torch.float16, False),
    (130, 2, 64, 0, torch.float32, False),     # one probe, no basis: mean shift only
    (4096, 8, 128, 64, torch.bfloat16, False),  # the multi-adapter bench's d = 1024 at its top rank
    (4096, 8, 128, 8, torch.bfloat16, True),
])
def test_kivi_subspace_matches_oracle(cuda, mode, n, n_kv, hd, r, fdt, inplace):
    gen = torch.Generator().manual_seed(n * 7 + r + (mode == "k"))
    cs = _case(gen, n, n_kv, hd, r, mode, probe_ratio=0.1 if r else 0.0)
    if fdt != torch.float32:  # the oracle sees exactly the values the kernel reads
        cs["fresh"] = cs["fresh"].to(fdt).float()
    base = _device_base(cs, cuda)
    out = None if inplace else K.KiviTensor.empty(n, cs["d"], mode, cuda)
    pb = K.SubspaceProblem(base=base, fresh=cs["fresh"].to(fdt).to(cuda), probe_index=cs["probes"].to(cuda),
                           basis=cs["B"].to(cuda) if cs["B"] is not None else None, rank=r, out=out)
    (o, sub, mu), = K.subspace_correct([pb], stats=True)
    torch.cuda.synchronize()
    _check(cs, o, sub, mu, (mode, n, r))


@pytest.mark.parametrize("mode", ["v", "k"])
@pytest.mark.parametrize("n,n_kv,hd,r,ratio", [
    (200, 8, 128, 16, 1.0),  # every token a probe: K rows all fresh (two staged per lane, the rest read
                             # directly), V rows all requantised from fresh on their own
    (333, 3, 64, 8, 0.6),    # d = 192 (6 blocks: V scale / zero read directly), a ragged last K group
])
def test_kivi_subspace_probe_heavy(cuda, mode, n, n_kv, hd, r, ratio):
    gen = torch.Generator().manual_seed(n + r + 17 * (mode == "k"))
    cs = _case(gen, n, n_kv, hd, r, mode, probe_ratio=ratio)
    cs["fresh"] = cs["fresh"].to(torch.bfloat16).float()
    out = K.KiviTensor.empty(n, cs["d"], mode, cuda)
    pb = K.SubspaceProblem(base=_device_base(cs, cuda), fresh=cs["fresh"].to(torch.bfloat16).to(cuda),
                           probe_index=cs["probes"].to(cuda), basis=cs["B"].to(cuda), rank=r, out=out)
    (o, sub, mu), = K.subspace_correct([pb], stats=True)
    torch.cuda.synchronize()
    _check(cs, o, sub, mu, ("probe-heavy", mode, n, ratio))


def test_kivi_subspace_batch_of_mixed_problems(cuda):
    """K and V views of several layers with different lengths and ranks in one call."""
    gen = torch.Generator().manual_seed(5)
    specs = [(500, 4, 64, 8, "v"), (500, 4, 64, 8, "k"), (97, 4, 64, 32, "v"), (64, 4, 64, 16, "k"),
             (1, 4, 64, 8, "v"), (333, 4, 64, 0, "k")]
    cases, probs = [], []
    for n, n_kv, hd, r, mode in specs:
        cs = _case(gen, n, n_kv, hd, r, mode)
        cases.append(cs)
        probs.append(K.SubspaceProblem(base=_device_base(cs, cuda), fresh=cs["fresh"].to(cuda),
                                       probe_index=cs["probes"].to(cuda),
                                       basis=cs["B"].to(cuda) if cs["B"] is not None else None, rank=r,
                                       out=K.KiviTensor.empty(n, cs["d"], mode, cuda)))
    res = K.subspace_correct(probs, stats=True)
    torch.cuda.synchronize()
    for i, (cs, (o, sub, mu)) in enumerate(zip(cases, res)):
        _check(cs, o, sub, mu, i)


def test_kivi_subspace_no_probes_and_svd_basis(cuda):
    gen = torch.Generator().manual_seed(6)
    # no probes: reference keeps reused (w * 0) -> output equals the requantised base
    cs = _case(gen, 200, 2, 64, 8, "v", probe_ratio=0.0)
    cs["probes"] = torch.zeros(0, dtype=torch.long)
    base = _device_base(cs, cuda)
    (o, _, _), = K.subspace_correct([K.SubspaceProblem(base=base, fresh=cs["fresh"].to(cuda),
                                                       probe_index=cs["probes"].to(cuda), basis=cs["B"].to(cuda),
                                                       rank=8, out=K.KiviTensor.empty(200, cs["d"], "v", cuda))])
    _check(cs, o, None, None, "no-probes")
    # K path with the basis from the probe residual's SVD (basis=None, rank=r): compare with
    # the oracle given the same basis
    cs = _case(gen, 400, 2, 64, 8, "k")
    base = _device_base(cs, cuda)
    fresh = cs["fresh"].to(cuda)
    res = K.probe_residual(base, fresh, cs["probes"].to(cuda))
    from deltakv_b200.subspace import svd_basis
    basis = svd_basis(res, 8)
    cs["B"] = basis.cpu()
    (o, sub, mu), = K.subspace_correct([K.SubspaceProblem(base=base, fresh=fresh, probe_index=cs["probes"].to(cuda),
                                                          basis=None, rank=8,
                                                          out=K.KiviTensor.empty(400, cs["d"], "k", cuda))],
                                       stats=True)
    _check(cs, o, sub, mu, "svd")


@pytest.mark.parametrize("fdt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d", [96, 1024])
def test_kivi_probe_residuals_batched(cuda, fdt, d):
    # one launch for several caches (both groupings, each job its own probe rows) equals the
    # oracle's fresh[P] - dequant(base)[P] exactly (fp32 subtraction of the same values)
    gen = torch.Generator().manual_seed(d + int(fdt == torch.float32))
    bases, freshes, probes, want = [], [], [], []
    n, m = 300, 37
    for j, mode in enumerate(("k", "v", "k", "v", "v")):
        x = torch.randn(n, d, generator=gen)
        c, s, z = OK.quantize(x.numpy(), mode)
        bases.append(K.KiviTensor(torch.from_numpy(c).to(cuda), torch.from_numpy(s).to(cuda),
                                  torch.from_numpy(z).to(cuda), mode))
        f = (x + 0.1 * torch.randn(n, d, generator=gen)).to(fdt)
        freshes.append(f.to(cuda))
        p = torch.randperm(n, generator=gen)[:m]
        probes.append(p.to(cuda))
        reused = OK.dequantize(c, s, z, mode)
        want.append(f.float().numpy()[p.numpy()] - reused[p.numpy()])
    got = K.probe_residuals(bases, freshes, probes).cpu().numpy()
    for j in range(len(bases)):
        np.testing.assert_array_equal(got[j], want[j])
        np.testing.assert_array_equal(got[j], K.probe_residual(bases[j], freshes[j], probes[j]).cpu().numpy())


@pytest.mark.parametrize("last_in_place", [True, False])
def test_kivi_subspace_views_pipelined_matches_sequential(cuda, last_in_place):
    # three adapter views over one shared int4 prefix (K bases from the probe residual, V the
    # adapter's B): the side-stream pipeline gives what view-by-view calls give (probe sums are
    # atomics, so up to float summation order) — with the last view correcting its own copy in
    # place and with every view writing its own output
    gen = torch.Generator().manual_seed(99)
    n, n_kv, hd = 512, 2, 64
    d = n_kv * hd
    shared = {m: _case(gen, n, n_kv, hd, 8, m) for m in ("k", "v")}

    def views():
        out = []
        for a in range(3):
            g = torch.Generator().manual_seed(1000 + a)
            probs = []
            probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.long), torch.randperm(n, generator=g)[:40]]))
            for m in ("k", "v"):
                cs = shared[m]
                base = _device_base(cs, cuda)
                fresh = (cs["fresh"] + 0.05 * torch.randn(n, d, generator=g)).to(torch.bfloat16).to(cuda)
                B = (torch.randn(d, 8, generator=g) / d ** 0.5).to(cuda)
                dst = None if a == 2 and last_in_place else K.KiviTensor.empty(n, d, m, cuda)
                probs.append(K.SubspaceProblem(base=base, fresh=fresh, probe_index=probes.to(cuda),
                                               basis=None if m == "k" else B, rank=8, out=dst))
            out.append(probs)
        return out

    seq = [[r[0] for r in K.subspace_correct(v)] for v in views()]
    pip = [[r[0] for r in rs] for rs in K.subspace_correct_views(views())]
    torch.cuda.synchronize()
    for a in range(3):
        for j in range(2):
            x, y = seq[a][j], pip[a][j]
            eq = (OK.unpack_nibbles(x.codes.cpu().numpy()) == OK.unpack_nibbles(y.codes.cpu().numpy())).mean()
            assert eq >= 0.999, (a, j, eq)
            torch.testing.assert_close(x.scale.float(), y.scale.float(), rtol=5e-3, atol=1e-6)


def test_kivi_subspace_views_edge_cases(cuda):
    assert K.subspace_correct_views([]) == []
    assert K.subspace_correct_views([[], []]) == [[], []]
    gen = torch.Generator().manual_seed(5)
    cs = _case(gen, 96, 2, 64, 8, "v")
    pb = lambda: K.SubspaceProblem(base=_device_base(cs, cuda), fresh=cs["fresh"].to(cuda),
                                   probe_index=cs["probes"].to(cuda), basis=cs["B"].to(cuda), rank=8,
                                   out=K.KiviTensor.empty(96, cs["d"], "v", cuda))
    (a,), = [[r[0] for r in K.subspace_correct([pb()])]]
    res = K.subspace_correct_views([[], [pb()]])
    assert res[0] == [] and len(res[1]) == 1
    torch.cuda.synchronize()
    eq = (OK.unpack_nibbles(a.codes.cpu().numpy()) == OK.unpack_nibbles(res[1][0][0].codes.cpu().numpy())).mean()
    assert eq >= 0.999
