"""The fused subspace iteration on an fp64 Gram matrix (``dkv_gram_subspace_iterate``) against
numpy, and :func:`gram_topr_basis` — the analytic route's rank truncation basis — against the
exact top-r eigen-subspace.

One step must be Cholesky QR of G Q to fp64 rounding (1e-9 of the largest entry; Q^T Q = I to
1e-10; the Rayleigh quotient Q^T G Q to 1e-10); several steps must span numpy's subspace
(projector difference 1e-8).  ``gram_topr_basis`` on a spectrum shaped like the propagated
ΔX (singular values 1 % apart at the cut): ||x (P - P_exact)||_F / ||x||_F <= 1e-6 without the
exact path; small / rank-deficient / degenerate inputs take the exact paths.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200 import _lib as L
from deltakv_b200 import ops

pytestmark = pytest.mark.gpu


def _iterate(g: np.ndarray, q0: np.ndarray, iters: int, cuda):
    d, k = q0.shape
    G = torch.from_numpy(np.ascontiguousarray(g)).to(cuda)
    Q = torch.from_numpy(np.ascontiguousarray(q0)).to(cuda)
    y = torch.empty(d, k, dtype=torch.float64, device=cuda)
    w = torch.empty(2, k, k, dtype=torch.float64, device=cuda)
    t = torch.empty(k, k, dtype=torch.float64, device=cuda)
    st = torch.empty(1, dtype=torch.int32, device=cuda)
    rc = L.lib().dkv_gram_subspace_iterate(G.data_ptr(), d, Q.data_ptr(), k, iters, y.data_ptr(), w.data_ptr(),
                                           t.data_ptr(), st.data_ptr(), ops.stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    return Q.cpu().numpy(), t.cpu().numpy(), y.cpu().numpy(), int(st.item())


def _gram(rng, m, d, decades=2.0):
    x = rng.standard_normal((m, d)) * np.logspace(0, -decades, d)
    g = x.T @ x
    return 0.5 * (g + g.T)


def _cholqr(y):
    r = np.linalg.cholesky(y.T @ y).T
    return np.linalg.solve(r.T, y.T).T


def test_one_step_is_cholesky_qr(cuda):
    rng = np.random.default_rng(0)
    d, k = 200, 40
    g = _gram(rng, 500, d)
    q0 = np.linalg.qr(rng.standard_normal((d, k)))[0]
    q, t, y, st = _iterate(g, q0, 1, cuda)
    assert st == 0
    want = _cholqr(g @ q0)
    assert np.abs(q - want).max() <= 1e-9 * np.abs(want).max()
    assert np.abs(q.T @ q - np.eye(k)).max() <= 1e-10
    rq = q.T @ g @ q
    assert np.abs(t - rq).max() <= 1e-10 * np.abs(rq).max()
    assert np.abs(y - g @ q).max() <= 1e-10 * np.abs(g @ q).max()


@pytest.mark.parametrize("d,k,iters", [(13, 5, 3), (96, 96, 2), (300, 72, 10), (577, 96, 6)])
def test_iterations_span_numpys_subspace(cuda, d, k, iters):
    rng = np.random.default_rng(d + k)
    g = _gram(rng, max(2 * d, 50), d, decades=1.0)
    q0 = rng.standard_normal((d, k))
    q, t, _, st = _iterate(g, q0, iters, cuda)
    assert st == 0
    want = q0
    for _ in range(iters):
        want = _cholqr(g @ want)
    assert np.abs(q @ q.T - want @ want.T).max() <= 1e-8
    assert np.abs(q.T @ q - np.eye(k)).max() <= 1e-9


def test_zero_steps_give_the_rayleigh_quotient_of_the_start(cuda):
    rng = np.random.default_rng(5)
    d, k = 150, 24
    g = _gram(rng, 300, d)
    q0 = np.linalg.qr(rng.standard_normal((d, k)))[0]
    q, t, _, st = _iterate(g, q0, 0, cuda)
    assert st == 0 and np.array_equal(q, q0)
    assert np.abs(t - q0.T @ g @ q0).max() <= 1e-10 * np.abs(t).max()


def test_a_block_that_lost_rank_is_flagged(cuda):
    rng = np.random.default_rng(6)
    x = rng.standard_normal((10, 100))  # G has rank 10 < k
    g = x.T @ x
    _, _, _, st = _iterate(0.5 * (g + g.T), rng.standard_normal((100, 32)), 1, cuda)
    assert st == 1


def test_invalid_arguments_are_rejected(cuda):
    z = torch.zeros(16, dtype=torch.float64, device=cuda)
    p = z.data_ptr()
    lib = L.lib()
    assert lib.dkv_gram_subspace_iterate(p, 8, p, 97, 1, p, p, p, p, ops.stream_ptr()) == L.DKV_ERR_INVALID_ARGUMENT
    assert lib.dkv_gram_subspace_iterate(p, 4, p, 5, 1, p, p, p, p, ops.stream_ptr()) == L.DKV_ERR_INVALID_ARGUMENT
    assert lib.dkv_gram_subspace_iterate(p, 8, p, 4, -1, p, p, p, p, ops.stream_ptr()) == L.DKV_ERR_INVALID_ARGUMENT


# singular values of the analytic route's propagated dX (SmolLM2-135M shape, 2048 tokens)
# at indices 0, 8, 16, 32, 48, 60, 63, 64, 65, 72, 80, 96, 128, 575
_PROFILE_AT = [0, 8, 16, 32, 48, 60, 63, 64, 65, 72, 80, 96, 128, 575]
_PROFILE = [1.0, 0.15, 0.09, 0.05, 0.037, 0.032, 0.0301, 0.0299, 0.0297, 0.026, 0.022, 0.017, 0.013, 0.004]


def _with_spectrum(m, d, s, seed):
    rng = np.random.default_rng(seed)
    u = np.linalg.qr(rng.standard_normal((m, d)))[0]
    v = np.linalg.qr(rng.standard_normal((d, d)))[0]
    return ((u * s) @ v.T).astype(np.float32)


def _exact_projector(x, r):
    g = x.astype(np.float64).T @ x.astype(np.float64)
    _, vec = np.linalg.eigh(g)
    v = vec[:, -r:]
    return v @ v.T


def _trunc_err(x, basis, r):
    x64 = x.astype(np.float64)
    b = basis.astype(np.float64)
    return np.linalg.norm(x64 @ (b @ b.T - _exact_projector(x, r))) / np.linalg.norm(x64)


def test_gram_topr_basis_on_a_gapless_spectrum(cuda, monkeypatch):
    import deltakv_b200.subspace as S

    exact_calls = []
    orig = S._eigh_top
    monkeypatch.setattr(S, "_eigh_top", lambda c, r: exact_calls.append(1) or orig(c, r))
    d, r = 576, 64
    s = np.interp(np.arange(d), _PROFILE_AT, _PROFILE)
    x = _with_spectrum(2048, d, s, 11)
    b = S.gram_topr_basis(torch.from_numpy(x).to(cuda), r).cpu().numpy()
    assert not exact_calls
    assert b.shape == (d, r)
    assert np.abs(b.T.astype(np.float64) @ b - np.eye(r)).max() <= 1e-6
    assert _trunc_err(x, b, r) <= 1e-6


def test_gram_topr_basis_small_and_rank_deficient_inputs(cuda):
    from deltakv_b200.subspace import gram_topr_basis

    rng = np.random.default_rng(12)
    for m, d, r in ((300, 64, 8), (50, 200, 16), (2000, 97, 40)):  # d <= 96: Jacobi on G; m < k: exact; d = 97: iteration
        x = (rng.standard_normal((m, d)) * np.logspace(0, -1.5, d)).astype(np.float32)
        b = gram_topr_basis(torch.from_numpy(x).to(cuda), r).cpu().numpy()
        assert b.shape == (d, r)
        assert _trunc_err(x, b, r) <= 1e-6


def test_gram_topr_basis_degenerate_and_zero_inputs(cuda):
    from deltakv_b200.subspace import gram_topr_basis

    d, r = 300, 32
    s = np.linspace(1.0, 0.1, d)
    s[r - 4: r + 4] = 0.5  # exactly repeated singular values across the cut
    x = _with_spectrum(600, d, s, 13)
    b = gram_topr_basis(torch.from_numpy(x).to(cuda), r).cpu().numpy().astype(np.float64)
    x64 = x.astype(np.float64)
    # any basis of a top-r subspace is optimal: the truncation error is the Eckart-Young one
    best = np.sqrt((np.linalg.svd(x64, compute_uv=False)[r:] ** 2).sum())
    assert abs(np.linalg.norm(x64 - x64 @ b @ b.T) - best) <= 1e-5 * best
    z = gram_topr_basis(torch.zeros(400, 200, device=cuda), 16)
    assert z.shape == (200, 16) and torch.isfinite(z).all()


def _gapless(cuda, seed=11):
    d = 576
    s = np.interp(np.arange(d), _PROFILE_AT, _PROFILE)
    x = _with_spectrum(2048, d, s, seed)
    return x, torch.from_numpy(x).to(cuda)


def test_gram_topr_basis_continues_by_the_predicted_steps(cuda, monkeypatch):
    # on this spectrum (subspace rate ~0.3 per step) 7 steps leave an estimate near 4e-4; the
    # Ritz values' rate predicts ~8 more, within twice the budget: one continuation, no exact
    # eigensolver, the same accuracy
    import deltakv_b200.subspace as S

    runs, exact = [], []
    orig_run, orig_exact = S._gram_run, S._eigh_top
    monkeypatch.setattr(S, "_gram_run", lambda job, n: runs.append(n) or orig_run(job, n))
    monkeypatch.setattr(S, "_eigh_top", lambda c, r: exact.append(1) or orig_exact(c, r))
    x, xd = _gapless(cuda)
    b = S.gram_topr_basis(xd, 64, iters=7).cpu().numpy()
    assert len(runs) == 2 and runs[0] == 7 and 0 < runs[1] <= 14 and not exact, runs
    assert _trunc_err(x, b, 64) <= 1e-6


def test_gram_topr_basis_falls_back_when_the_prediction_is_too_long(cuda, monkeypatch):
    # 2 steps: the predicted continuation (~11) exceeds twice the budget, the exact path is taken
    import deltakv_b200.subspace as S

    exact = []
    orig_exact = S._eigh_top
    monkeypatch.setattr(S, "_eigh_top", lambda c, r: exact.append(1) or orig_exact(c, r))
    x, xd = _gapless(cuda)
    b = S.gram_topr_basis(xd, 64, iters=2).cpu().numpy()
    assert exact == [1]
    assert _trunc_err(x, b, 64) <= 1e-7  # the exact basis, rounded to fp32


def test_analytic_loop_graphs_survive_fallbacks(cuda, monkeypatch):
    # a tolerance no estimate meets: every truncation continues then takes the exact path, in
    # the eager call and in graph replays; the replays' captured flags are restored each time
    import types

    import deltakv_b200.analytic as A
    import deltakv_b200.subspace as S
    from deltakv_b200.rope import RotaryEmbedding

    g = torch.Generator(device=cuda).manual_seed(5)
    d, dff, H, Hkv, hd, n, L_ = 128, 256, 4, 2, 32, 256, 4
    rnd = lambda *s_, sc=0.05: torch.randn(*s_, generator=g, device=cuda) * sc
    mod = lambda w: types.SimpleNamespace(weight=w)
    blocks = [types.SimpleNamespace(attn_norm=mod(1 + rnd(d)), mlp_norm=mod(1 + rnd(d)), q_proj=mod(rnd(H * hd, d)),
                                    k_proj=mod(rnd(Hkv * hd, d)), v_proj=mod(rnd(Hkv * hd, d)),
                                    o_proj=mod(rnd(d, H * hd)), gate_proj=mod(rnd(dff, d)), up_proj=mod(rnd(dff, d)),
                                    down_proj=mod(rnd(d, dff))) for _ in range(L_)]
    cfg = types.SimpleNamespace(n_heads=H, n_kv_heads=Hkv, head_dim=hd, d_model=d, rms_eps=1e-5)
    model = types.SimpleNamespace(cfg=cfg, blocks=blocks, rope=RotaryEmbedding(hd, max_seq=n, base=10000.0))
    from deltakv_b200.types import LayerDelta, LowRankFactors

    lora = lambda fin, fout: LowRankFactors(A=rnd(4, fin, sc=fin ** -0.5), B=rnd(fout, 4, sc=1.0), scale=0.05)
    delta = types.SimpleNamespace(layers={l: LayerDelta(layer_idx=l, projections={
        "q_proj": lora(d, H * hd), "k_proj": lora(d, Hkv * hd), "v_proj": lora(d, Hkv * hd),
        "o_proj": lora(H * hd, d)}) for l in range(L_)})
    conf = types.SimpleNamespace(hidden_stride=2, propagator_rank=16)
    h = [torch.randn(n, d, generator=g, device=cuda) for _ in range(L_)]
    hm = [torch.randn(n, d, generator=g, device=cuda) for _ in range(L_)]
    hidden = types.SimpleNamespace(layer_in=lambda l: h[l], layer_mid=lambda l: hm[l], seq_len=n)
    monkeypatch.setattr(A, "USE_GRAPHS", False)
    want = A.analytic_patches(hidden, delta, model, conf)
    monkeypatch.setattr(A, "USE_GRAPHS", True)
    monkeypatch.setattr(S, "GRAM_TOL", 1e-300)
    for _ in range(4):  # eager, eager + capture, then two replays
        got = A.analytic_patches(hidden, delta, model, conf)
        for l in range(L_):
            assert want[l].k_dense.norm() > 0 and want[l].v_dense.norm() > 0
            assert ((got[l].k_dense - want[l].k_dense).norm() / want[l].k_dense.norm()).item() < 1e-5, l
            assert ((got[l].v_dense - want[l].v_dense).norm() / want[l].v_dense.norm()).item() < 1e-5, l
