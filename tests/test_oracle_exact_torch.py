"""The torch CPU form of the exact branch (the timed CPU baseline) against the numpy oracle."""
import numpy as np
import torch

from oracle import exact as OX
from oracle import exact_torch as OT
from oracle.numerics import bf16_bits_to_f32


def _case(seq, d, n_kv, hd, r, bs, kind, seed=0):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(seq, d, generator=g) * (0.5 + torch.rand(seq, 1, generator=g))
    sc = (h.abs().amax(-1) / 448.0).float()
    if kind == "e4m3":
        xb = (h / sc[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        xb = (h / sc[:, None]).to(torch.float16)
    w = 1.0 + 0.05 * torch.randn(d, generator=g)
    fk = (torch.randn(r, d, generator=g) / d ** 0.5, torch.randn(n_kv * hd, r, generator=g), 0.25)
    fv = (torch.randn(r, d, generator=g) / d ** 0.5, torch.randn(n_kv * hd, r, generator=g), 0.25)
    nblk = (seq + bs - 1) // bs + 3
    table = torch.from_numpy(np.random.default_rng(seed).permutation(nblk).astype(np.int64))
    pages = torch.randn(nblk, bs, n_kv, hd, generator=g).to(torch.bfloat16)
    return xb, sc, w, fk, fv, table, pages


def _run_both(seq, d, n_kv, hd, r, bs, kind, theta=10000.0):
    xb, sc, w, fk, fv, table, pages = _case(seq, d, n_kv, hd, r, bs, kind)
    cos_h, sin_h = OX.rope_tables(hd, seq, theta)
    # torch form
    x = OT.dequant_x(xb, kind, sc)
    xn = OT.rmsnorm(x, w, 1e-5)
    rope = OT.rope_full(torch.from_numpy(cos_h), torch.from_numpy(sin_h), seq)
    dk_t, dv_t = OT.exact_kv_delta(xn, fk, fv, n_kv, hd, rope)
    kp_t = pages.clone()
    OT.scatter_into_paged(dk_t, kp_t, table, bs)
    # numpy oracle
    xo = OX.dequant_x(xb.numpy(), kind, sc.numpy())
    xno = OX.rmsnorm(xo, w.numpy(), 1e-5)
    fko = tuple(t.numpy() if torch.is_tensor(t) else t for t in fk)
    fvo = tuple(t.numpy() if torch.is_tensor(t) else t for t in fv)
    dk_o, dv_o = OX.exact_kv_delta(xno, fko, fvo, n_kv, hd, (cos_h, sin_h))
    kp_o = pages.view(torch.uint16).numpy().copy()
    OX.scatter_into_paged(dk_o, kp_o, table.tolist(), bs, kind="bf16")
    return (dk_t.numpy(), dv_t.numpy(), kp_t.float().numpy()), (dk_o, dv_o, bf16_bits_to_f32(kp_o))


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_exact_torch_matches_oracle_fp8():
    (dk, dv, kp), (dk_o, dv_o, kp_o) = _run_both(seq=100, d=256, n_kv=2, hd=64, r=8, bs=16, kind="e4m3",
                                                 theta=500000.0)
    assert _rel(dk, dk_o) < 1e-5 and _rel(dv, dv_o) < 1e-5
    # pages: round_bf16(page + delta) — equal except where the fp32 sums straddle a bf16 tie
    assert np.mean(kp == kp_o) > 0.999
    assert _rel(kp, kp_o) < 1e-4


def test_exact_torch_matches_oracle_f16_ragged():
    (dk, dv, kp), (dk_o, dv_o, kp_o) = _run_both(seq=37, d=128, n_kv=1, hd=32, r=4, bs=8, kind="f16")
    assert _rel(dk, dk_o) < 1e-5 and _rel(dv, dv_o) < 1e-5
    assert np.mean(kp == kp_o) > 0.999


def test_exact_torch_short_table():
    xb, sc, w, fk, fv, table, pages = _case(40, 64, 1, 16, 2, 8, "f16")
    delta = torch.zeros(40, 1, 16)
    try:
        OT.scatter_into_paged(delta, pages, table[:2], 8)
    except ValueError as e:
        assert "block_table shorter than prefix" in str(e)
    else:
        raise AssertionError("expected ValueError")
