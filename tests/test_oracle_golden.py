"""Pin the CPU oracle to golden vectors produced by the reference implementation."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import exact as OX
from oracle.numerics import bf16_bits_to_f32, e4m3_bits_to_f32, f32_to_bf16_bits, f32_to_e4m3_bits
from tests.conftest import golden


def test_bf16_rounding_matches_torch():
    import torch

    x = torch.randn(10000, dtype=torch.float32) * 1e3
    x[:10] = torch.tensor([0.0, -0.0, 1.0, 1.00390625, 1.005859375, 3.0e38, -3.0e38, 1e-40, 65504.0, 2.0 ** -130])
    ours = f32_to_bf16_bits(x.numpy())
    ref = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)
    assert np.array_equal(bf16_bits_to_f32(ref), x.to(torch.bfloat16).float().numpy())


def test_e4m3_decode_and_encode_match_torch():
    import torch

    bits = torch.arange(256, dtype=torch.uint8)
    ref = bits.view(torch.float8_e4m3fn).float().numpy()
    ours = e4m3_bits_to_f32(bits.numpy())
    finite = ~np.isnan(ref)
    assert np.array_equal(ours[finite], ref[finite])
    assert np.isnan(ours[~finite]).all()
    x = (torch.randn(20000) * 100).clamp(-448, 448)
    x[:6] = torch.tensor([0.0, 448.0, -448.0, 0.0009765625, 0.001953125 * 1.5, 17.0])
    assert np.array_equal(f32_to_e4m3_bits(x.numpy()), x.to(torch.float8_e4m3fn).view(torch.uint8).numpy())


def test_paged_roundtrip_golden():
    g = golden("paged")
    cache = np.zeros((8, 8, 2, 8), np.float32)
    OX.scatter_into_paged(g["rt_delta"], cache, list(g["rt_table"]), 8)
    assert np.array_equal(cache, g["rt_cache_out"])
    got = OX.gather_from_paged(cache, list(g["rt_table"]), 20, 8)
    assert np.array_equal(got, g["rt_gather"])
    assert np.allclose(got, g["rt_delta"])


@pytest.mark.parametrize("name", ["l4", "l5a", "l5b"])
def test_paged_bf16_layouts_golden(name):
    g = golden("paged")
    c = g[f"{name}_in"].copy()
    OX.scatter_into_paged(g[f"{name}_delta"], c, list(g["l_table"]), int(g["l_bs"]), kv_dim=int(g[f"{name}_kv"]), kind="bf16")
    assert np.array_equal(c, g[f"{name}_out"])  # bit-exact
    got = OX.gather_from_paged(c, list(g["l_table"]), 13, int(g["l_bs"]), kv_dim=int(g[f"{name}_kv"]))
    assert np.array_equal(got, g[f"{name}_gather"])


def test_paged_errors_match_reference_text():
    with pytest.raises(ValueError, match="block_table shorter than prefix"):
        OX.scatter_into_paged(np.zeros((20, 1, 4), np.float32), np.zeros((4, 8, 1, 4), np.float32), [0, 1], 8)
    with pytest.raises(ValueError, match="unsupported paged KV layout"):
        OX.scatter_into_paged(np.zeros((4, 1, 4), np.float32), np.zeros((3, 4, 8, 1, 4), np.float32), [0], 8)


def test_rope_tables_match_reference():
    g = golden("config1")
    cos, sin = OX.rope_tables(int(g["hd"]), g["rope_cos"].shape[0])
    assert np.abs(cos - g["rope_cos"]).max() <= 2e-7
    assert np.abs(sin - g["rope_sin"]).max() <= 2e-7


def test_layer0_exact_golden():
    g = golden("layer0")
    n_kv, hd = int(g["n_kv"]), int(g["hd"])
    rope = (g["rope_cos"], g["rope_sin"])
    dk, dv = OX.exact_kv_delta(g["xn"], (g["a_k"], g["b_k"], float(g["s_k"])),
                               (g["a_v"], g["b_v"], float(g["s_v"])), n_kv, hd, rope)
    assert np.abs(dk - g["dk"]).max() < 1e-6
    assert np.abs(dv - g["dv"]).max() < 1e-6
    kp = g["k0"] + dk
    assert np.abs(kp - g["k_patched"]).max() < 1e-6
    # the reference's own claim: layer-0 patch equals the fresh prefill (<2e-5)
    assert np.abs(kp - g["k_fresh"]).max() < 2e-5
    assert np.abs(g["v0"] + dv - g["v_fresh"]).max() < 2e-5


def test_config1_exact_golden():
    g = golden("config1")
    n_kv, hd = int(g["n_kv"]), int(g["hd"])
    rope = (g["rope_cos"], g["rope_sin"])
    for l in range(g["h_in"].shape[0]):
        xn = OX.rmsnorm(g["h_in"][l], g["norm_w"][l], float(g["eps"]))
        assert np.abs(xn - g["xn"][l]).max() < 1e-5
        sk, sv = g["scales"][l]
        dk, dv = OX.exact_kv_delta(xn, (g["a_k"][l], g["b_k"][l], float(sk)), (g["a_v"][l], g["b_v"][l], float(sv)),
                                   n_kv, hd, rope)
        assert np.abs(dk - g["dk"][l]).max() < 1e-6
        assert np.abs(dv - g["dv"][l]).max() < 1e-6
    # paged bf16 through the permuted table: bit-exact given the reference's dK/dV
    bs = int(g["block_size"])
    for l in range(g["h_in"].shape[0]):
        kp = g["k_pages_in"][l].copy()
        OX.scatter_into_paged(g["dk"][l], kp, list(g["block_table"]), bs, kind="bf16")
        assert np.array_equal(kp, g["k_pages_out"][l])


def test_fp8_paged_golden():
    g = golden("fp8_paged")
    n_kv, hd = int(g["n_kv"]), int(g["hd"])
    L_ = g["x_bits"].shape[0]
    kp = [g["k_pages_in"][l].copy() for l in range(L_)]
    vp = [g["v_pages_in"][l].copy() for l in range(L_)]
    factors = [((g["a_k"][l], g["b_k"][l], float(g["s_k"])), (g["a_v"][l], g["b_v"][l], float(g["s_v"]))) for l in range(L_)]
    OX.exact_patch_paged(x=g["x_bits"], x_dtype="e4m3", x_scale=g["x_scale"], norm_w=g["norm_w"], eps=float(g["eps"]),
                         factors=factors, cu_seqlens=g["cu_seqlens"], block_tables=g["block_tables"], k_pages=kp,
                         v_pages=vp, n_kv=n_kv, hd=hd, rope=(g["rope_cos"], g["rope_sin"]), kind="bf16")
    for l in range(L_):
        for ours, ref in ((kp[l], g["k_pages_out"][l]), (vp[l], g["v_pages_out"][l])):
            a, b = bf16_bits_to_f32(ours), bf16_bits_to_f32(ref)
            rel = np.linalg.norm(a - b) / np.linalg.norm(b)
            assert rel < 1e-5
            # fp32 summation order may flip a bf16 rounding; almost every element is identical
            assert (ours == ref).mean() > 0.995


def test_config1_logits_and_kl_golden():
    from oracle.model import logits_from_kv, next_token_kl, weights_from_golden

    g = golden("config1")
    w = weights_from_golden(g)
    kw = dict(n_layers=g["h_in"].shape[0], n_heads=int(g["n_heads"]), n_kv=int(g["n_kv"]), hd=int(g["hd"]),
              eps=float(g["eps"]), rope=(g["rope_cos"], g["rope_sin"]))
    fresh = logits_from_kv(w, g["tokens"], g["k_fresh"], g["v_fresh"], **kw)
    patched = logits_from_kv(w, g["tokens"], g["k_patched"], g["v_patched"], **kw)
    assert np.abs(fresh - g["fresh_logits"]).max() < 1e-5
    assert np.abs(patched - g["patched_logits"]).max() < 1e-5
    assert abs(next_token_kl(fresh, patched) - float(g["kl_ref"])) < 1e-6


@pytest.mark.parametrize("case", ["t1", "t2", "v", "k"])
def test_subspace_golden(case):
    from oracle.subspace import subspace_correct

    g = golden("subspace")
    basis = None
    if case == "t1" or (case in ("v", "k") and int(g[f"{case}_use_basis"])):
        basis = g[f"{case}_basis"]
    corr, sub, orth = subspace_correct(g[f"{case}_reused"], g[f"{case}_fresh"], g[f"{case}_probes"], basis=basis,
                                       rank=int(g[f"{case}_rank"]))
    ref = g[f"{case}_corr"]
    assert np.linalg.norm(corr - ref) / np.linalg.norm(ref) < 1e-5
    assert np.abs(orth - g[f"{case}_orth"]).max() < 1e-4 * (1 + np.abs(g[f"{case}_orth"]).max())
    assert np.abs(sub - g[f"{case}_sub"]).max() < 1e-4 * (1 + np.abs(g[f"{case}_sub"]).max())


def test_kivi_spec_vs_reference_fake_quant():
    """The stored format differs from _minmax_quantize only by fp16 storage of scale/zero."""
    from oracle import kivi as OK

    g = golden("kivi")
    xv = g["xv"].reshape(70, -1)
    c, s, z = OK.quantize(xv, "v")
    deq = OK.dequantize(c, s, z, "v")
    ref = g["xv_q"].reshape(70, -1)
    step = (xv.reshape(70, -1, 32).max(-1) - xv.reshape(70, -1, 32).min(-1)) / 15
    # fp16 scale/zero move a value into the neighbouring bin only near a bin boundary:
    # at most one step away from the reference's fp32 fake-quant, almost always within 1%
    err = np.abs(deq - ref).reshape(70, -1, 32) / step[..., None]
    assert err.max() <= 1.01 and (err < 1e-2).mean() > 0.98
    xk = g["xk"].reshape(96, -1)
    c, s, z = OK.quantize(xk, "k")
    deqk = OK.dequantize(c, s, z, "k")
    refk = g["xk_q"].reshape(96, -1)
    stepk = (xk.max() - xk.min()) / 15
    assert np.abs(deqk - refk).max() <= 1.01 * stepk and (np.abs(deqk - refk) < 1e-2 * stepk).mean() > 0.98


def test_kivi_roundtrip_properties():
    from oracle import kivi as OK

    rng = np.random.default_rng(0)
    for mode in ("v", "k"):
        x = rng.standard_normal((77, 96)).astype(np.float32)
        c, s, z = OK.quantize(x, mode)
        deq = OK.dequantize(c, s, z, mode)
        c2, s2, z2 = OK.quantize(deq, mode)  # idempotent on its own output up to fp16 re-rounding
        assert np.abs(OK.dequantize(c2, s2, z2, mode) - deq).max() < 2e-2
        assert np.abs(deq - x).max() <= (x.max() - x.min()) / 15
        assert np.array_equal(OK.unpack_nibbles(OK.pack_nibbles(OK.unpack_nibbles(c))), OK.unpack_nibbles(c))


def test_dense_paged_golden():
    """The dense route's oracle (A=dW, B=I through the exact route) against the reference."""
    from oracle import dense as OD

    g = golden("dense_paged")
    n_kv, hd = int(g["n_kv"]), int(g["hd"])
    L_ = g["x_bits"].shape[0]
    kp = [g["k_pages_in"][l].copy() for l in range(L_)]
    vp = [g["v_pages_in"][l].copy() for l in range(L_)]
    OD.dense_patch_paged(x=bf16_bits_to_f32(g["x_bits"]), norm_w=g["norm_w"], eps=float(g["eps"]),
                         dw_k=bf16_bits_to_f32(g["dw_k_bits"]), dw_v=bf16_bits_to_f32(g["dw_v_bits"]),
                         cu_seqlens=g["cu_seqlens"], block_tables=g["block_tables"], k_pages=kp, v_pages=vp,
                         n_kv=n_kv, hd=hd, rope=(g["rope_cos"], g["rope_sin"]), kind="bf16")
    for l in range(L_):
        for ours, ref, base in ((kp[l], g["k_pages_out"][l], g["k_pages_in"][l]),
                                (vp[l], g["v_pages_out"][l], g["v_pages_in"][l])):
            a, b = bf16_bits_to_f32(ours), bf16_bits_to_f32(ref)
            assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-5
            assert (ours == ref).mean() > 0.995
            assert not np.array_equal(ref, base)  # the case patches something


def test_measured_error_golden():
    from oracle.metrics import measured_error

    g = golden("errors")
    rel, per = measured_error(g["pk"], g["pv"], g["fk"], g["fv"])
    assert np.allclose(per, g["per_layer"], rtol=1e-5, atol=1e-9)
    assert abs(rel - float(g["rel"])) <= 1e-5 * float(g["rel"])


def test_analytic_oracle_golden():
    # the fp64 restatement of the analytic route against the reference's fp32 run
    from oracle import analytic as OA
    from tests._analytic_golden import load, rel

    g, W, Ls, cfg = load()
    for l, (dk, dv) in enumerate(OA.analytic_patches(g["h"], g["h_mid"], W, Ls, cfg)):
        assert rel(dk, g["dk"][l]) < 1e-5 and rel(dv, g["dv"][l]) < 1e-5, l
    cos, sin = OA.rope_tables(cfg["hd"], g["h"].shape[1], cfg["rope_base"])
    y, dy = OA.rmsnorm_first_order(g["h"][1], g["dx1"], W[1]["attn_norm"], cfg["eps"])
    assert rel(y, g["rn_y"]) < 1e-6 and rel(dy, g["rn_dy"]) < 1e-6
    dh, dk, dv = OA.attention_first_order(g["rn_y"], g["rn_dy"], W[1]["q"], W[1]["k"], W[1]["v"], W[1]["o"], Ls[1],
                                          cfg["n_heads"], cfg["n_kv"], cfg["hd"], cos, sin)
    assert max(rel(dh, g["at_dh"]), rel(dk, g["at_dk"]), rel(dv, g["at_dv"])) < 1e-6
    ym, dym = OA.rmsnorm_first_order(g["h_mid"][1], g["dx1"], W[1]["mlp_norm"], cfg["eps"])
    assert rel(OA.mlp_first_order(ym, dym, W[1]["gate"], W[1]["up"], W[1]["down"], Ls[1]), g["ml_out"]) < 1e-6


def test_compare_kv_golden():
    # the reference computes in fp32: its cosine of identical tensors is 0.99999976, so the
    # fp64 restatement agrees to 1e-6
    from oracle.metrics import compare_kv

    g = golden("compare")
    rows, mx, mean, mn = compare_kv(g["pk"], g["pv"], g["fk"], g["fv"])
    np.testing.assert_allclose(rows, g["per_layer"], rtol=0, atol=1e-6)
    assert abs(mx - float(g["max_rel"])) <= 1e-6 and abs(mean - float(g["mean_rel"])) <= 1e-6
    assert abs(mn - float(g["min_cos"])) <= 1e-6


def _replay_chain(g):
    chain = []
    for si in range(2):
        stage = {}
        for key in list(g.keys()):
            if key.startswith(f"s{si}_l"):
                l = int(key.split("_")[1][1:])
                nm = key.split("_", 2)[2]
                stage.setdefault(l, {})[nm] = g[key]
        chain.append(stage)
    return chain


def test_probe_and_replay_oracle_golden():
    from oracle import probe as OP

    g = golden("probe")
    sc = OP.weight_axis_scores(g["x_norm"], [(g["a_k"], float(g["s_k"])), (g["a_v"], float(g["s_v"]))])
    assert np.allclose(sc, g["scores"], rtol=1e-5, atol=1e-6)
    assert np.array_equal(OP.select_probes(g["scores"], 0.15, 4, 0.5), g["probes"])
    ko, vo, extra = OP.apply_probe_to_cache(
        g["base_k"], g["base_v"], {l: (g["fresh_k"][l], g["fresh_v"][l]) for l in range(2)}, g["probes"], 0.15, 0.40,
        v_bases={0: g["b_v"], 1: g["b_v"]}, k_ranks={0: g["b_k"].shape[1], 1: g["b_k"].shape[1]}, subspace_rank=4,
        probe_layers={0})
    assert np.array_equal(extra, g["extra"])
    assert np.abs(ko - g["out_k"]).max() < 1e-4 and np.abs(vo - g["out_v"]).max() < 1e-4
    gate = OP.residual_gate(g["base_k"][0], g["out_k"][0], g["fresh_k"][0], g["probes"], 0.15, 0.40)
    assert np.array_equal(np.sort(gate), np.sort(g["gate"]))

    r = golden("replay")
    k, v = OP.replay(r["base_k"], r["base_v"], _replay_chain(r))
    assert np.abs(k - r["out_k"]).max() < 1e-5 and np.abs(v - r["out_v"]).max() < 1e-5


def _smol_patched(w, dl, h, k, v):
    """The oracle's exact branch on the SmolLM2-shaped stack: RMSNorm -> exact_kv_delta (k/v
    factors) added to the cached K/V."""
    from tests import _smol_model as SM

    tabs = OX.rope_tables(SM.HD, SM.SEQ, SM.ROPE_BASE)
    kp, vp = k.copy(), v.copy()
    for l in range(SM.N_LAYERS):
        xn = OX.rmsnorm(h[l], w[f"blocks_{l}_attn_norm_weight"], SM.EPS)
        dk, dv = OX.exact_kv_delta(xn, dl[l]["k_proj"], dl[l]["v_proj"], SM.N_KV, SM.HD, tabs)
        kp[l] += dk
        vp[l] += dv
    return kp, vp


def test_smol_prefill_and_kl_golden():
    """The oracle prefill and exact branch at the SmolLM2-135M shape (4 of 30 layers, 2048
    tokens) against the reference's own run; also the size of the error that storing the
    patched cache in bf16 pages adds to the next-token distribution."""
    from oracle import model as OM
    from tests import _smol_model as SM

    g = golden("smol_kl")
    assert np.array_equal(g["tokens"], SM.tokens())
    w = SM.weights()
    dl = SM.delta(w)
    kw = dict(n_layers=SM.N_LAYERS, n_heads=SM.N_HEADS, n_kv=SM.N_KV, hd=SM.HD, eps=SM.EPS,
              rope=OX.rope_tables(SM.HD, SM.SEQ, SM.ROPE_BASE))
    _, k, v, h = OM.prefill(w, g["tokens"], **kw)
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    # fp32 summation order (2048-key softmax sums, 576/1536-long products) differs from torch's:
    # ~1e-5 relative after four blocks
    assert rel(h[:, :4], g["h_head"]) < 5e-5 and rel(h[:, -4:], g["h_tail"]) < 5e-5
    assert rel(k[:, -4:], g["k_tail"]) < 5e-5 and rel(v[:, -4:], g["v_tail"]) < 5e-5
    norms = lambda t: np.array([np.linalg.norm(t[l].astype(np.float64)) for l in range(t.shape[0])])
    for got, key in ((h, "h_norms"), (k, "k_norms"), (v, "v_norms")):
        assert np.allclose(norms(got), g[key], rtol=1e-5)
    kp, vp = _smol_patched(w, dl, h, k, v)
    assert np.allclose(norms(kp), g["patched_k_norms"], rtol=1e-5)
    assert np.allclose(norms(vp), g["patched_v_norms"], rtol=1e-5)
    w1 = SM.merged(w, dl)
    logits = OM.logits_from_kv(w1, g["tokens"], kp, vp, **kw)
    assert OM.next_token_kl(g["patched_logits"], logits) < 1e-8
    assert abs(OM.next_token_kl(g["fresh_logits"], logits) - float(g["kl_ref"])) < 1e-6
    # the same cache rounded to bf16 pages: bf16 storage alone moves the next-token
    # distribution by ~4e-8 nats, the floor of the GPU test's 1e-6 bound
    kb = bf16_bits_to_f32(f32_to_bf16_bits(kp)).reshape(kp.shape)
    vb = bf16_bits_to_f32(f32_to_bf16_bits(vp)).reshape(vp.shape)
    lb = OM.logits_from_kv(w1, g["tokens"], kb, vb, **kw)
    assert OM.next_token_kl(g["patched_logits"], lb) < 2e-7


def test_smol_dense_route_golden():
    """The oracle's dense route (exact_kv_delta with A=dW, B=I) on the SmolLM2-shaped stack
    against the reference's run (tests/golden/smol_dense.npz)."""
    from oracle import dense as OD
    from oracle import model as OM
    from tests import _smol_model as SM

    g = golden("smol_dense")
    w = SM.weights()
    dd = SM.dense_delta(w)
    tabs = OX.rope_tables(SM.HD, SM.SEQ, SM.ROPE_BASE)
    kw = dict(n_layers=SM.N_LAYERS, n_heads=SM.N_HEADS, n_kv=SM.N_KV, hd=SM.HD, eps=SM.EPS, rope=tabs)
    _, k, v, h = OM.prefill(w, g["tokens"], **kw)
    for l in range(SM.N_LAYERS):
        xn = OX.rmsnorm(h[l], w[f"blocks_{l}_attn_norm_weight"], SM.EPS)
        dk, dv = OX.exact_kv_delta(xn, *OD.dense_factors(dd[l]["k_proj"], dd[l]["v_proj"]), SM.N_KV, SM.HD, tabs)
        k[l] += dk
        v[l] += dv
    logits = OM.logits_from_kv(SM.merged_dense(w, dd), g["tokens"], k, v, **kw)
    assert OM.next_token_kl(g["patched_logits"], logits) < 1e-8
    assert abs(OM.next_token_kl(g["fresh_logits"], logits) - float(g["kl_ref"])) < 1e-6
