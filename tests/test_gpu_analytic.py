"""Analytic route (Route A) on the GPU against the reference's golden run
(tests/golden/analytic.npz: GQA toy, LoRA on every projection of layers 0-2) and the fp64
oracle.

Tolerances (relative L2): the module functions on layer 1 within 1e-5 of the reference (fp32
arithmetic, summation order differs); the engine loop's per-layer ΔK / ΔV within 1e-4 (four
layers of propagation through the rank-8 truncation); the attention core against the oracle on
the same (possibly bf16-rounded) inputs within 1e-5 (fp32 arithmetic in both).
"""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from deltakv_b200 import analytic as A
from deltakv_b200.rope import RotaryEmbedding
from deltakv_b200.types import LayerDelta, LowRankFactors
from oracle import analytic as OA
from tests._analytic_golden import PROJ, load, rel

pytestmark = pytest.mark.gpu


def _layers(Ls, dev):
    out = {}
    for l, facs in Ls.items():
        proj = {f"{p}_proj": LowRankFactors(A=torch.from_numpy(a).to(dev), B=torch.from_numpy(b).to(dev), scale=s)
                for p, (a, b, s) in facs.items()}
        out[l] = LayerDelta(layer_idx=l, projections=proj)
    return out


def _model(W, cfg, dev):
    t = lambda a: torch.from_numpy(np.asarray(a)).to(dev)
    mod = lambda a: types.SimpleNamespace(weight=t(a))
    blocks = []
    for w in W:
        b = types.SimpleNamespace(attn_norm=mod(w["attn_norm"]), mlp_norm=mod(w["mlp_norm"]))
        for p in PROJ:
            setattr(b, f"{p}_proj", mod(w[p]))
        blocks.append(b)
    mcfg = types.SimpleNamespace(n_heads=cfg["n_heads"], n_kv_heads=cfg["n_kv"], head_dim=cfg["hd"],
                                 d_model=cfg["d_model"], rms_eps=cfg["eps"])
    return types.SimpleNamespace(cfg=mcfg, blocks=blocks,
                                 rope=RotaryEmbedding(cfg["hd"], max_seq=cfg["rope_max"], base=cfg["rope_base"]))


def test_module_functions_match_reference(cuda):
    g, W, Ls, cfg = load()
    t = lambda a: torch.from_numpy(np.asarray(a)).to(cuda)
    layers = _layers(Ls, cuda)
    y, dy = A.rmsnorm_first_order(t(g["h"][1]), t(g["dx1"]), t(W[1]["attn_norm"]), cfg["eps"])
    assert rel(y.cpu(), g["rn_y"]) < 1e-6 and rel(dy.cpu(), g["rn_dy"]) < 1e-6
    rope = RotaryEmbedding(cfg["hd"], max_seq=cfg["rope_max"], base=cfg["rope_base"])
    dh, dk, dv, attn = A.attention_first_order(t(g["rn_y"]), t(g["rn_dy"]), t(W[1]["q"]), t(W[1]["k"]), t(W[1]["v"]),
                                               t(W[1]["o"]), layers[1], n_heads=cfg["n_heads"],
                                               n_kv_heads=cfg["n_kv"], head_dim=cfg["hd"], rope=rope)
    assert attn is None
    assert rel(dh.cpu(), g["at_dh"]) < 1e-5
    assert rel(dk.cpu(), g["at_dk"]) < 1e-5 and rel(dv.cpu(), g["at_dv"]) < 1e-5
    ym, dym = A.rmsnorm_first_order(t(g["h_mid"][1]), t(g["dx1"]), t(W[1]["mlp_norm"]), cfg["eps"])
    out = A.mlp_first_order(ym, dym, t(W[1]["gate"]), t(W[1]["up"]), t(W[1]["down"]), layers[1])
    assert rel(out.cpu(), g["ml_out"]) < 1e-5


def test_engine_loop_matches_reference(cuda):
    g, W, Ls, cfg = load()
    model = _model(W, cfg, cuda)
    h = [torch.from_numpy(x).to(cuda) for x in g["h"]]
    hm = [torch.from_numpy(x).to(cuda) for x in g["h_mid"]]
    hidden = types.SimpleNamespace(layer_in=lambda l: h[l], layer_mid=lambda l: hm[l], seq_len=h[0].shape[0])
    delta = types.SimpleNamespace(layers=_layers(Ls, cuda))
    conf = types.SimpleNamespace(hidden_stride=cfg["hidden_stride"], propagator_rank=cfg["propagator_rank"])
    patches = A.analytic_patches(hidden, delta, model, conf)
    for l in range(len(W)):
        assert rel(patches[l].k_dense.cpu(), g["dk"][l]) < 1e-4, l
        assert rel(patches[l].v_dense.cpu(), g["dv"][l]) < 1e-4, l


def test_engine_loop_replays_as_graphs_and_recaptures(cuda, monkeypatch):
    # after the first call each layer is a CUDA graph replay: the same patches as the eager path
    # (to the atomics' summation order) for this and another sequence; an in-place weight
    # update is detected and re-captured
    g, W, Ls, cfg = load()
    model = _model(W, cfg, cuda)
    h = [torch.from_numpy(x).to(cuda) for x in g["h"]]
    hm = [torch.from_numpy(x).to(cuda) for x in g["h_mid"]]
    snap = lambda hh, mm: types.SimpleNamespace(layer_in=lambda l: hh[l], layer_mid=lambda l: mm[l],
                                                seq_len=hh[0].shape[0])
    delta = types.SimpleNamespace(layers=_layers(Ls, cuda))
    conf = types.SimpleNamespace(hidden_stride=cfg["hidden_stride"], propagator_rank=cfg["propagator_rank"])
    other = snap([x * 0.5 + 0.1 for x in h], [x.flip(0) for x in hm])

    def eager(hidden):
        monkeypatch.setattr(A, "USE_GRAPHS", False)
        out = A.analytic_patches(hidden, delta, model, conf)
        monkeypatch.setattr(A, "USE_GRAPHS", True)
        return out

    for _ in range(2):  # eager; eager, then captured
        A.analytic_patches(snap(h, hm), delta, model, conf)
    sets = [v for k, v in A._graph_sets.items() if k[0] == id(model) and k[1] == id(delta)]
    assert sets and sets[0], "the layers were not captured"
    for hidden in (snap(h, hm), other):
        want, got = eager(hidden), A.analytic_patches(hidden, delta, model, conf)
        for l in range(len(W)):
            assert rel(got[l].k_dense.cpu(), want[l].k_dense.cpu()) < 1e-6, l
            assert rel(got[l].v_dense.cpu(), want[l].v_dense.cpu()) < 1e-6, l
    replayed = A.analytic_patches(snap(h, hm), delta, model, conf)
    for l in range(len(W)):
        assert rel(replayed[l].k_dense.cpu(), g["dk"][l]) < 1e-4, l
    model.blocks[0].q_proj.weight.mul_(1.01)
    want, got = eager(snap(h, hm)), A.analytic_patches(snap(h, hm), delta, model, conf)
    for l in range(len(W)):
        assert rel(got[l].k_dense.cpu(), want[l].k_dense.cpu()) < 1e-6, l
    after = A.analytic_patches(snap(h, hm), delta, model, conf)  # the re-captured graphs
    for l in range(len(W)):
        assert rel(after[l].v_dense.cpu(), want[l].v_dense.cpu()) < 1e-6, l


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,H,Hkv,hd", [(300, 8, 2, 64), (129, 4, 4, 128), (70, 6, 3, 32), (33, 2, 1, 16)])
def test_attention_core_matches_oracle(cuda, dtype, n, H, Hkv, hd):
    gen = torch.Generator().manual_seed(n + hd)
    mk = lambda h: (torch.randn(n, h, hd, generator=gen) * 0.7).to(dtype)
    q, dq, k, dk, v, dv = mk(H), 0.1 * mk(H), mk(Hkv), 0.1 * mk(Hkv), mk(Hkv), 0.1 * mk(Hkv)
    ctx, dctx = A.attention_core(*(x.to(cuda) for x in (q, dq, k, dk, v, dv)), want_ctx=True)
    qn, dqn, kn, dkn, vn, dvn = (x.double().numpy() for x in (q, dq, k, dk, v, dv))
    rep = H // Hkv
    kf, dkf, vf, dvf = (np.repeat(x, rep, axis=1) for x in (kn, dkn, vn, dvn))
    s = np.einsum("qhd,khd->hqk", qn, kf) * hd ** -0.5 + np.triu(np.full((n, n), -np.inf), 1)
    a = np.exp(s - s.max(-1, keepdims=True))
    a /= a.sum(-1, keepdims=True)
    ds = (np.einsum("qhd,khd->hqk", dqn, kf) + np.einsum("qhd,khd->hqk", qn, dkf)) * hd ** -0.5
    da = a * (ds - (a * ds).sum(-1, keepdims=True))
    want_ctx = np.einsum("hqk,khd->qhd", a, vf)
    want_dctx = np.einsum("hqk,khd->qhd", da, vf) + np.einsum("hqk,khd->qhd", a, dvf)
    assert rel(ctx.cpu(), want_ctx) < 1e-5
    assert rel(dctx.cpu(), want_dctx) < 1e-5


def test_rank_truncate_is_the_best_rank_r_approximation(cuda):
    gen = torch.Generator().manual_seed(9)
    d = torch.randn(200, 6, generator=gen) @ torch.randn(6, 96, generator=gen) + 0.01 * torch.randn(200, 96, generator=gen)
    codes, basis = A.rank_truncate(d.to(cuda), 6)
    want = OA.rank_truncate(d.double().numpy(), 6)
    assert rel((codes @ basis.T).cpu(), want) < 1e-5
    assert codes.shape == (200, 6) and basis.shape == (96, 6)
