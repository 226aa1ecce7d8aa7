"""The torch fp32 form of the analytic route (the timed CPU baseline) against the fp64 numpy oracle."""
import numpy as np
import torch

from oracle import analytic as OA
from oracle import analytic_torch as OAT


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def test_analytic_torch_matches_oracle():
    rng = np.random.default_rng(0)
    L, n, d, H, Hkv, hd, ff, r = 3, 48, 64, 4, 2, 16, 96, 4
    rnd = lambda *s, sc=0.1: rng.standard_normal(s) * sc  # noqa: E731
    W = [{"q": rnd(H * hd, d), "k": rnd(Hkv * hd, d), "v": rnd(Hkv * hd, d), "o": rnd(d, H * hd),
          "gate": rnd(ff, d), "up": rnd(ff, d), "down": rnd(d, ff),
          "attn_norm": 1 + rnd(d), "mlp_norm": 1 + rnd(d)} for _ in range(L)]
    Ls = {l: {p: (rnd(r, fi, sc=fi ** -0.5), rnd(fo, r, sc=1.0), 0.05)
              for p, (fi, fo) in (("q", (d, H * hd)), ("k", (d, Hkv * hd)), ("v", (d, Hkv * hd)), ("o", (H * hd, d)),
                                  ("gate", (d, ff)), ("up", (d, ff)), ("down", (ff, d)))} for l in range(L)}
    # propagator rank = d: the truncation keeps everything, so fp32 and fp64 SVDs agree
    cfg = dict(n_heads=H, n_kv=Hkv, hd=hd, d_model=d, eps=1e-5, rope_base=10000.0, hidden_stride=2,
               propagator_rank=d)
    h, hm = rng.standard_normal((L, n, d)), rng.standard_normal((L, n, d))
    ref = OA.analytic_patches(h, hm, W, Ls, cfg)
    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.float32)  # noqa: E731
    Wt = [{k: t(v) for k, v in w.items()} for w in W]
    Lt = {l: {p: (t(a), t(b), s) for p, (a, b, s) in f.items()} for l, f in Ls.items()}
    got = OAT.analytic_patches(t(h), t(hm), Wt, Lt, cfg)
    for (dk, dv), (rk, rv) in zip(got, ref):
        assert _rel(dk.numpy(), rk.reshape(dk.shape)) < 1e-4
        assert _rel(dv.numpy(), rv.reshape(dv.shape)) < 1e-4


def test_rank_truncate_torch_with_gap():
    rng = np.random.default_rng(1)
    u = np.linalg.qr(rng.standard_normal((64, 8)))[0]
    v = np.linalg.qr(rng.standard_normal((32, 8)))[0]
    m = (u * np.array([8, 7, 6, 5, 1e-3, 1e-3, 1e-3, 1e-3])) @ v.T
    got = OAT.rank_truncate(torch.tensor(m, dtype=torch.float32), 4).numpy()
    assert _rel(got, OA.rank_truncate(m, 4)) < 1e-5
