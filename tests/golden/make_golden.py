"""Generate golden vectors by running the reference implementation (adityaraj-09/DeltaKV).

Run in the build container, where the reference source is available:

    python tests/golden/make_golden.py <reference checkout>/src [case ...]

It imports the reference read-only (no bytecode written), drives its own functions on
seeded inputs and stores inputs and outputs as ``tests/golden/*.npz``.  The tests read
only the .npz files, so they run where the reference is absent.

Cases:
  paged.npz        scatter_into_paged / gather_from_paged: the reference's own
                   test_paged_roundtrip case (tests/test_engine.py:184-191) plus bf16
                   caches in the three layouts of paged.py:18-37.
  layer0.npz       the setup of tests/test_layer1_exact.py:37-55 (exact_kv_patch on
                   layer 0 of the conftest toy, then apply_layer_patches, vs a fresh
                   prefill under the new weights).
  config1.npz      the CPU-toy configuration: 4 layers, d=64, GQA 4/2, 64 tokens, rank-4
                   k/v LoRA on every layer at relative scale 0.01 -> rmsnorm_tensors ->
                   zeroth_order_patches -> apply_layer_patches, fresh prefill, logits, KL,
                   and the same patch scattered into bf16 pages through a permuted table.
  fp8_paged.npz    ragged multi-sequence batch: fp8-e4m3 stored activations with per-token
                   scales, RMSNorm with non-unit weight, ranks k=8 / v=16, RoPE, bf16 pages,
                   computed per (layer, sequence) with the reference's RMSNorm,
                   exact_kv_patch, materialize and scatter_into_paged.
  subspace.npz     subspace_correct with a given basis (V path), with basis=None (K path,
                   SVD of the probe residual) and the reference tests' two cases
                   (tests/test_quality.py:32-64).
  dense_paged.npz  dense weight delta (full-rank dW_K, dW_V, as an RL step produces) through
                   the reference's exact route with LowRankFactors(A=dW, B=I, scale=1):
                   RMSNorm, exact_kv_patch, materialize, scatter_into_paged over a ragged
                   batch of bf16 activations into bf16 pages.
  probe.npz        weight_axis_scores + select_probes on a LoRA delta, residual_gate, and
                   apply_probe_to_cache over two layers (gated and ungated) with LoRA bases.
  replay.npz       the engine's replay loop (engine.py:205-210): base KV plus a two-stage chain
                   of apply_layer_patches (codes @ basis patches, then dense patches).
  errors.npz       patches.compose.measured_error of a patched vs a fresh KVCache (per layer).
  compare.npz      metrics.compare_kv of the same pair (per-layer relative L2 and cosine).
  analytic.npz     the analytic route on a GQA toy (4 layers, d=64, 4/2 heads, 48 tokens) with
                   rank-4 LoRA on every projection of layers 0-2: the engine's per-layer loop
                   (engine.py:377-432, hidden_stride 2, propagator_rank 8) and, on layer 1 with a
                   seeded dx, rmsnorm_first_order, attention_first_order and mlp_first_order.
  kivi.npz         metrics._minmax_quantize (4 bits, group 32) on the last dimension (the
                   per-token V grouping) and on the transposed tensor (per-channel K
                   grouping), plus kivi_noise_floor on a small KVCache.
  engine.npz       DeltaKVEngine end to end on the CPU toy (4 layers, d=64, GQA 4/2, 64
                   tokens, rank-4 q/k/v LoRA at scale 0.01 as the reference's `bench`
                   command builds it): prefill, commit_delta, evaluate_against_fresh for
                   route exact, hybrid and subspace (the probe route with
                   apply_probe_to_cache(..., probe_layers=set())), with the arguments and
                   results of every hot-path call the engine made (recorded by wrapping the
                   engine module's names), the report, and DeltaKVConnector.patch_paged of the
                   exact view into bf16 paged caches.
  smol_dense.npz   the same stack with a full-rank dW on k/v of every layer (relative norm 0.02,
                   bf16 values) through the reference's exact route with A=dW, B=I: fresh,
                   patched and stale last-token logits and their KL.
  smol_kl.npz      SmolLM2-135M-shaped decoder (tests/_smol_model.py: seeded weights, 4 of
                   30 layers, 2048 tokens, rank-8 q/k/v/o LoRA at relative norm 0.01): the
                   reference's prefill, rmsnorm_tensors -> zeroth_order_patches ->
                   apply_layer_patches, apply_delta, fresh prefill, last-token logits of the
                   fresh and patched caches, next_token_kl, and pins of the prefill (rows and
                   norms of the stored activations and K/V).

Usage: ``make_golden.py <reference>/src`` writes every file; ``make_golden.py <reference>/src
engine smol_kl`` only the named ones (``core`` = the files above engine.npz).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

sys.dont_write_bytecode = True
OUT = Path(__file__).resolve().parent


def bf16_bits(t) -> np.ndarray:
    import torch

    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def core_cases(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    import torch

    from deltakv.deltas.descriptor import LayerDelta, lora_layer
    from deltakv.deltas.factors import LowRankFactors, random_lora_factors
    from deltakv.deltas.lora import lora_delta
    from deltakv.metrics import next_token_kl
    from deltakv.model import RMSNorm, ToyConfig, ToyTransformer
    from deltakv.paged import gather_from_paged, scatter_into_paged
    from deltakv.patches.compose import apply_layer_patches
    from deltakv.patches.exact import exact_kv_patch, zeroth_order_patches
    from deltakv.patches.subspace import subspace_correct
    from deltakv.rope import RotaryEmbedding
    from deltakv.types import WeightVersion

    torch.set_num_threads(4)
    torch.set_grad_enabled(False)

    # ------------------------------------------------------------------ paged
    g = torch.Generator().manual_seed(0)
    paged = {}
    seq, h, d, bs = 20, 2, 8, 8
    delta = torch.randn(seq, h, d, generator=g)
    cache = torch.zeros(8, bs, h, d)
    table = [3, 1, 5]
    scatter_into_paged(delta, cache, table, bs)
    paged["rt_delta"] = delta.numpy()
    paged["rt_table"] = np.array(table, np.int32)
    paged["rt_cache_out"] = cache.numpy()
    paged["rt_gather"] = gather_from_paged(cache, table, seq, bs).numpy()
    # bf16 caches in the three layouts
    nb, bs2, seq2 = 9, 4, 13
    table2 = [7, 2, 0, 5]
    for name, shape, kv in (
        ("l4", (nb, bs2, h, d), 0),
        ("l5a", (2, nb, bs2, h, d), 1),
        ("l5b", (nb, 2, bs2, h, d), 0),
    ):
        c = torch.randn(*shape, generator=g).to(torch.bfloat16)
        dl = torch.randn(seq2, h, d, generator=g) * 0.01
        paged[f"{name}_in"] = bf16_bits(c)
        paged[f"{name}_delta"] = dl.numpy()
        scatter_into_paged(dl, c, table2, bs2, kv_dim=kv)
        paged[f"{name}_out"] = bf16_bits(c)
        paged[f"{name}_kv"] = np.int32(kv)
        paged[f"{name}_gather"] = bf16_bits(gather_from_paged(c, table2, seq2, bs2, kv_dim=kv))
    paged["l_table"] = np.array(table2, np.int32)
    paged["l_bs"] = np.int32(bs2)
    np.savez_compressed(OUT / "paged.npz", **paged)

    # ----------------------------------------------------------------- layer0
    torch.manual_seed(0)
    toy = ToyTransformer(ToyConfig(n_layers=4, d_model=64, n_heads=4, n_kv_heads=4, d_ff=128, vocab_size=128))
    tokens = torch.arange(48) % toy.cfg.vocab_size
    _, kv0, hidden = toy.prefill(tokens)
    gl = torch.Generator().manual_seed(1)
    c = toy.cfg
    fk = random_lora_factors(c.d_model, c.n_kv_heads * c.head_dim, 4, scale=0.05, generator=gl, name="k_proj")
    fv = random_lora_factors(c.d_model, c.n_kv_heads * c.head_dim, 4, scale=0.05, generator=gl, name="v_proj")
    delta = lora_delta(source=WeightVersion(id="base"), target=WeightVersion(id="lora", parent_id="base", kind="lora"),
                       layers={0: lora_layer(0, k=fk, v=fv)})
    with torch.no_grad():
        xn = toy.blocks[0].attn_norm(hidden.layer_in(0))
        patch = exact_kv_patch(xn, delta.layers[0], n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, rope=toy.rope)
        dk, dv = patch.materialize(c.n_kv_heads, c.head_dim)
        patched = apply_layer_patches(kv0, {0: patch})
        toy.apply_delta(delta, version=WeightVersion(id="lora"))
        _, kv1, _ = toy.prefill(tokens)
    hd = c.head_dim
    np.savez_compressed(
        OUT / "layer0.npz",
        xn=xn.numpy(), a_k=fk.A.numpy(), b_k=fk.B.numpy(), s_k=np.float32(fk.scale),
        a_v=fv.A.numpy(), b_v=fv.B.numpy(), s_v=np.float32(fv.scale),
        rope_cos=toy.rope.cos_cached[:, : hd // 2].numpy(), rope_sin=toy.rope.sin_cached[:, : hd // 2].numpy(),
        dk=dk.numpy(), dv=dv.numpy(), k0=kv0.k[0].numpy(), v0=kv0.v[0].numpy(),
        k_patched=patched.k[0].numpy(), v_patched=patched.v[0].numpy(),
        k_fresh=kv1.k[0].numpy(), v_fresh=kv1.v[0].numpy(), n_kv=np.int32(c.n_kv_heads), hd=np.int32(hd),
    )

    # ---------------------------------------------------------------- config1
    torch.manual_seed(0)
    cfg = ToyConfig(n_layers=4, d_model=64, n_heads=4, n_kv_heads=2, d_ff=128, vocab_size=256)
    model = ToyTransformer(cfg)
    gt = torch.Generator().manual_seed(0)
    tokens = torch.randint(0, 256, (64,), generator=gt)
    with torch.no_grad():
        logits0, kv_base, hidden = model.prefill(tokens)
    gf = torch.Generator().manual_seed(1)
    d_kv = cfg.n_kv_heads * cfg.head_dim
    layers, A_k, B_k, A_v, B_v, S = {}, [], [], [], [], []
    for i, blk in enumerate(model.blocks):
        facs = {}
        for name, lin in (("k", blk.k_proj), ("v", blk.v_proj)):
            A = torch.randn(4, cfg.d_model, generator=gf) / cfg.d_model ** 0.5
            B = torch.randn(d_kv, 4, generator=gf)
            rel = 0.01 * lin.weight.norm() / (B @ A).norm()
            facs[name] = LowRankFactors(A=A, B=B, scale=float(rel), name=f"{name}_proj")
        layers[i] = lora_layer(i, k=facs["k"], v=facs["v"])
        A_k.append(facs["k"].A.numpy()); B_k.append(facs["k"].B.numpy())
        A_v.append(facs["v"].A.numpy()); B_v.append(facs["v"].B.numpy())
        S.append((facs["k"].scale, facs["v"].scale))
    delta = lora_delta(source=WeightVersion(id="base"), target=WeightVersion(id="lora", parent_id="base", kind="lora"),
                       layers=layers)
    with torch.no_grad():
        xn = model.rmsnorm_tensors(hidden)
        patches = zeroth_order_patches(xn, delta, n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, rope=model.rope)
        patched = apply_layer_patches(kv_base, patches)
        deltas = {l: p.materialize(cfg.n_kv_heads, cfg.head_dim) for l, p in patches.items()}
        model.apply_delta(delta, version=WeightVersion(id="lora"))
        fresh_logits, kv_fresh, _ = model.prefill(tokens)
        patched_logits = model.logits_from_kv(tokens, patched)
        kl_ref = next_token_kl(fresh_logits, patched_logits)
        kl_stale = next_token_kl(fresh_logits, model.logits_from_kv(tokens, kv_base))
    # bf16 pages through a permuted block table (seed 2)
    bs = 16
    gp = torch.Generator().manual_seed(2)
    nblk = 12
    perm = torch.randperm(nblk, generator=gp)[: (64 + bs - 1) // bs].tolist()
    k_pages_in, v_pages_in, k_pages_out, v_pages_out = [], [], [], []
    for l in range(cfg.n_layers):
        kp = torch.randn(nblk, bs, cfg.n_kv_heads, cfg.head_dim, generator=gp).to(torch.bfloat16)
        vp = torch.randn(nblk, bs, cfg.n_kv_heads, cfg.head_dim, generator=gp).to(torch.bfloat16)
        # the cached prefix itself
        for i in range(64):
            kp[perm[i // bs], i % bs] = kv_base.k[l, i].to(torch.bfloat16)
            vp[perm[i // bs], i % bs] = kv_base.v[l, i].to(torch.bfloat16)
        k_pages_in.append(bf16_bits(kp)); v_pages_in.append(bf16_bits(vp))
        scatter_into_paged(deltas[l][0], kp, perm, bs)
        scatter_into_paged(deltas[l][1], vp, perm, bs)
        k_pages_out.append(bf16_bits(kp)); v_pages_out.append(bf16_bits(vp))
    hd = cfg.head_dim
    np.savez_compressed(
        OUT / "config1.npz",
        tokens=tokens.numpy().astype(np.int64),
        h_in=np.stack([h.numpy() for h in hidden.h]),
        norm_w=np.stack([b.attn_norm.weight.detach().numpy() for b in model.blocks]),
        eps=np.float32(cfg.rms_eps),
        a_k=np.stack(A_k), b_k=np.stack(B_k), a_v=np.stack(A_v), b_v=np.stack(B_v),
        scales=np.array(S, np.float32),
        rope_cos=model.rope.cos_cached[:, : hd // 2].numpy(), rope_sin=model.rope.sin_cached[:, : hd // 2].numpy(),
        xn=np.stack([xn[l].numpy() for l in range(cfg.n_layers)]),
        dk=np.stack([deltas[l][0].numpy() for l in range(cfg.n_layers)]),
        dv=np.stack([deltas[l][1].numpy() for l in range(cfg.n_layers)]),
        k_base=kv_base.k.numpy(), v_base=kv_base.v.numpy(),
        k_patched=patched.k.numpy(), v_patched=patched.v.numpy(),
        k_fresh=kv_fresh.k.numpy(), v_fresh=kv_fresh.v.numpy(),
        patched_logits=patched_logits.numpy(), fresh_logits=fresh_logits.view(-1, cfg.vocab_size)[-1].numpy(),
        kl_ref=np.float64(kl_ref), kl_stale=np.float64(kl_stale),
        block_table=np.array(perm, np.int32), block_size=np.int32(bs),
        k_pages_in=np.stack(k_pages_in), v_pages_in=np.stack(v_pages_in),
        k_pages_out=np.stack(k_pages_out), v_pages_out=np.stack(v_pages_out),
        n_kv=np.int32(cfg.n_kv_heads), hd=np.int32(hd),
        n_heads=np.int32(cfg.n_heads), rope_base=np.float32(cfg.rope_base),
        **{f"w_{k.replace('.', '_')}": v.detach().numpy() for k, v in model.state_dict().items()},
    )

    # -------------------------------------------------------------- fp8_paged
    g8 = torch.Generator().manual_seed(3)
    L_, dm, n_kv, hd, bs = 2, 128, 2, 64, 16
    lens = [37, 16, 1, 70, 133]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    rows = int(cu[-1])
    rope = RotaryEmbedding(hd, max_seq=512, base=10000.0)
    x = torch.randn(L_, rows, dm, generator=g8) * 3.0
    amax = x.abs().amax(dim=-1).clamp_min(1e-12)
    xscale = (amax / 448.0).float()
    xq = (x / xscale[..., None]).to(torch.float8_e4m3fn)
    xdq = xq.float() * xscale[..., None]
    norm_w = 1.0 + 0.1 * torch.randn(L_, dm, generator=g8)
    rk, rv = 8, 16
    a_k = torch.randn(L_, rk, dm, generator=g8) / dm ** 0.5
    b_k = torch.randn(L_, n_kv * hd, rk, generator=g8)
    a_v = torch.randn(L_, rv, dm, generator=g8) / dm ** 0.5
    b_v = torch.randn(L_, n_kv * hd, rv, generator=g8)
    s_k, s_v = 0.02, 0.015
    max_blocks = max((n + bs - 1) // bs for n in lens)
    nblk = sum((n + bs - 1) // bs for n in lens) + 3
    perm = torch.randperm(nblk, generator=g8).tolist()
    tables = np.full((len(lens), max_blocks), -1, np.int32)
    k = 0
    for b, n in enumerate(lens):
        for i in range((n + bs - 1) // bs):
            tables[b, i] = perm[k]
            k += 1
    kp_in = [torch.randn(nblk, bs, n_kv, hd, generator=g8).to(torch.bfloat16) for _ in range(L_)]
    vp_in = [torch.randn(nblk, bs, n_kv, hd, generator=g8).to(torch.bfloat16) for _ in range(L_)]
    kp_out = [t.clone() for t in kp_in]
    vp_out = [t.clone() for t in vp_in]
    for l in range(L_):
        norm = RMSNorm(dm, 1e-6)
        with torch.no_grad():
            norm.weight.copy_(norm_w[l])
        ld = LayerDelta(layer_idx=l, projections={
            "k_proj": LowRankFactors(A=a_k[l], B=b_k[l], scale=s_k),
            "v_proj": LowRankFactors(A=a_v[l], B=b_v[l], scale=s_v),
        })
        for b, n in enumerate(lens):
            with torch.no_grad():
                xn_b = norm(xdq[l, cu[b]:cu[b + 1]])
                p = exact_kv_patch(xn_b, ld, n_kv_heads=n_kv, head_dim=hd, rope=rope)
                dk, dv = p.materialize(n_kv, hd)
            t = tables[b, : (n + bs - 1) // bs].tolist()
            scatter_into_paged(dk, kp_out[l], t, bs)
            scatter_into_paged(dv, vp_out[l], t, bs)
    np.savez_compressed(
        OUT / "fp8_paged.npz",
        x_bits=xq.view(torch.uint8).numpy(), x_scale=xscale.numpy(), norm_w=norm_w.numpy(), eps=np.float32(1e-6),
        a_k=a_k.numpy(), b_k=b_k.numpy(), a_v=a_v.numpy(), b_v=b_v.numpy(), s_k=np.float32(s_k), s_v=np.float32(s_v),
        cu_seqlens=cu, block_tables=tables, block_size=np.int32(bs),
        rope_cos=rope.cos_cached[:, : hd // 2].numpy(), rope_sin=rope.sin_cached[:, : hd // 2].numpy(),
        k_pages_in=np.stack([bf16_bits(t) for t in kp_in]), v_pages_in=np.stack([bf16_bits(t) for t in vp_in]),
        k_pages_out=np.stack([bf16_bits(t) for t in kp_out]), v_pages_out=np.stack([bf16_bits(t) for t in vp_out]),
        n_kv=np.int32(n_kv), hd=np.int32(hd),
    )

    # ------------------------------------------------------------ dense_paged
    gd = torch.Generator().manual_seed(7)
    L_, dm, n_kv, hd, bs = 2, 256, 2, 128, 16
    lens = [37, 128, 1, 200, 300]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    rows = int(cu[-1])
    rope = RotaryEmbedding(hd, max_seq=512, base=500000.0)
    x = (torch.randn(L_, rows, dm, generator=gd) * 2.0).to(torch.bfloat16).float()  # stored bf16 X
    norm_w = 1.0 + 0.1 * torch.randn(L_, dm, generator=gd)
    d_kv = n_kv * hd
    # deltas of a few percent of the cached values (an RL step's is ~1e-3 of W)
    dw_k = (torch.randn(L_, d_kv, dm, generator=gd) * 0.003).to(torch.bfloat16).float()
    dw_v = (torch.randn(L_, d_kv, dm, generator=gd) * 0.003).to(torch.bfloat16).float()
    max_blocks = max((n + bs - 1) // bs for n in lens)
    nblk = sum((n + bs - 1) // bs for n in lens) + 5
    perm = torch.randperm(nblk, generator=gd).tolist()
    tables = np.full((len(lens), max_blocks), -1, np.int32)
    k = 0
    for b, n in enumerate(lens):
        for i in range((n + bs - 1) // bs):
            tables[b, i] = perm[k]
            k += 1
    kp_in = [torch.randn(nblk, bs, n_kv, hd, generator=gd).to(torch.bfloat16) for _ in range(L_)]
    vp_in = [torch.randn(nblk, bs, n_kv, hd, generator=gd).to(torch.bfloat16) for _ in range(L_)]
    kp_out = [t.clone() for t in kp_in]
    vp_out = [t.clone() for t in vp_in]
    eye = torch.eye(d_kv)
    for l in range(L_):
        norm = RMSNorm(dm, 1e-6)
        with torch.no_grad():
            norm.weight.copy_(norm_w[l])
        ld = LayerDelta(layer_idx=l, projections={
            "k_proj": LowRankFactors(A=dw_k[l], B=eye, scale=1.0),
            "v_proj": LowRankFactors(A=dw_v[l], B=eye, scale=1.0),
        })
        for b, n in enumerate(lens):
            with torch.no_grad():
                xn_b = norm(x[l, cu[b]:cu[b + 1]])
                p = exact_kv_patch(xn_b, ld, n_kv_heads=n_kv, head_dim=hd, rope=rope)
                dk, dv = p.materialize(n_kv, hd)
            t = tables[b, : (n + bs - 1) // bs].tolist()
            scatter_into_paged(dk, kp_out[l], t, bs)
            scatter_into_paged(dv, vp_out[l], t, bs)
    np.savez_compressed(
        OUT / "dense_paged.npz",
        x_bits=bf16_bits(x), norm_w=norm_w.numpy(), eps=np.float32(1e-6),
        dw_k_bits=bf16_bits(dw_k), dw_v_bits=bf16_bits(dw_v),
        cu_seqlens=cu, block_tables=tables, block_size=np.int32(bs),
        rope_cos=rope.cos_cached[:, : hd // 2].numpy(), rope_sin=rope.sin_cached[:, : hd // 2].numpy(),
        k_pages_in=np.stack([bf16_bits(t) for t in kp_in]), v_pages_in=np.stack([bf16_bits(t) for t in vp_in]),
        k_pages_out=np.stack([bf16_bits(t) for t in kp_out]), v_pages_out=np.stack([bf16_bits(t) for t in vp_out]),
        n_kv=np.int32(n_kv), hd=np.int32(hd),
    )

    # --------------------------------------------------------------- subspace
    sub = {}
    torch.manual_seed(0)
    seq, h, d, r = 32, 2, 8, 3
    reused = torch.randn(seq, h, d)
    basis = torch.randn(h * d, r)
    codes = torch.randn(seq, r) * 0.05
    mu = torch.randn(h * d)
    gram_mu = torch.linalg.lstsq(basis, mu.unsqueeze(-1)).solution.squeeze(-1)
    mu = mu - basis @ gram_mu
    fresh = reused + (codes @ basis.T).view(seq, h, d) + mu.view(1, h, d)
    probes = torch.arange(0, 16)
    corr, subsp, orth = subspace_correct(reused, fresh, probes, basis=basis, rank=r)
    sub.update(t1_reused=reused.numpy(), t1_fresh=fresh.numpy(), t1_probes=probes.numpy(), t1_basis=basis.numpy(),
               t1_rank=np.int32(r), t1_corr=corr.numpy(), t1_sub=subsp.numpy(), t1_orth=orth.numpy())
    torch.manual_seed(1)
    reused = torch.randn(24, 2, 4)
    mu = torch.randn(2, 4)
    fresh = reused + mu
    probes = torch.tensor([0, 2, 4, 6, 8, 10])
    corr, subsp, orth = subspace_correct(reused, fresh, probes, basis=None, rank=1)
    sub.update(t2_reused=reused.numpy(), t2_fresh=fresh.numpy(), t2_probes=probes.numpy(), t2_rank=np.int32(1),
               t2_corr=corr.numpy(), t2_sub=subsp.numpy(), t2_orth=orth.numpy())
    # larger V-path (given basis) and K-path (SVD basis) cases with structure + drift
    gs = torch.Generator().manual_seed(4)
    for tag, n, nkv, hdim, rr, use_basis in (("v", 300, 4, 32, 8, True), ("k", 300, 4, 32, 8, False)):
        dkv = nkv * hdim
        reused = torch.randn(n, nkv, hdim, generator=gs)
        B = torch.randn(dkv, rr, generator=gs)
        cds = torch.randn(n, rr, generator=gs) * 0.1
        drift = torch.randn(dkv, generator=gs) * 0.05
        noise = torch.randn(n, dkv, generator=gs) * 0.01
        fresh = reused + (cds @ B.T + drift + noise).view(n, nkv, hdim)
        probes = torch.unique(torch.randperm(n, generator=gs)[:30].sort().values)
        probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.long), probes]))
        corr, subsp, orth = subspace_correct(reused, fresh, probes, basis=B if use_basis else None, rank=rr)
        sub.update({f"{tag}_reused": reused.numpy(), f"{tag}_fresh": fresh.numpy(), f"{tag}_probes": probes.numpy(),
                    f"{tag}_basis": B.numpy(), f"{tag}_use_basis": np.int32(use_basis), f"{tag}_rank": np.int32(rr),
                    f"{tag}_corr": corr.numpy(), f"{tag}_sub": subsp.numpy(), f"{tag}_orth": orth.numpy()})
    np.savez_compressed(OUT / "subspace.npz", **sub)

    # ----------------------------------------------------------------- errors
    from deltakv.patches.compose import measured_error
    from deltakv.patches.tensors import KVCache as RefKV

    ge = torch.Generator().manual_seed(8)
    fk, fv = torch.randn(3, 50, 2, 16, generator=ge), torch.randn(3, 50, 2, 16, generator=ge)
    pk = fk + 0.01 * torch.randn(3, 50, 2, 16, generator=ge) * torch.tensor([1.0, 3.0, 0.0]).view(3, 1, 1, 1)
    pv = fv + 0.02 * torch.randn(3, 50, 2, 16, generator=ge)
    est = measured_error(RefKV(k=pk, v=pv, version=WeightVersion(id="p")), RefKV(k=fk, v=fv, version=WeightVersion(id="f")))
    np.savez_compressed(OUT / "errors.npz", pk=pk.numpy(), pv=pv.numpy(), fk=fk.numpy(), fv=fv.numpy(),
                        per_layer=np.array(est.per_layer, np.float64), rel=np.float64(est.relative_kv_l2))

    # --------------------------------------------------------------- analytic
    import types as _types

    from deltakv.deltas.factors import random_lora_factors
    from deltakv.engine import DeltaKVEngine
    from deltakv.patches.analytic import attention_first_order, mlp_first_order, rmsnorm_first_order

    torch.manual_seed(3)
    acfg = ToyConfig(n_layers=4, d_model=64, n_heads=4, n_kv_heads=2, d_ff=128, vocab_size=256)
    amodel = ToyTransformer(acfg)
    ga = torch.Generator().manual_seed(5)
    atok = torch.randint(0, 256, (48,), generator=ga)
    with torch.no_grad():
        _, _, ahidden = amodel.prefill(atok)
    dkv_ = acfg.n_kv_heads * acfg.head_dim
    dq_ = acfg.n_heads * acfg.head_dim
    shapes = {"q": (acfg.d_model, dq_), "k": (acfg.d_model, dkv_), "v": (acfg.d_model, dkv_),
              "o": (dq_, acfg.d_model), "gate": (acfg.d_model, acfg.d_ff), "up": (acfg.d_model, acfg.d_ff),
              "down": (acfg.d_ff, acfg.d_model)}
    alayers, fac_arrays = {}, {}
    for li in (0, 1, 2):
        kw = {}
        for nm, (fin, fout) in shapes.items():
            f = random_lora_factors(fin, fout, 4, scale=0.05, generator=ga, name=f"{nm}_proj")
            kw[nm] = f
            fac_arrays[f"lora_{li}_{nm}_A"] = f.A.numpy()
            fac_arrays[f"lora_{li}_{nm}_B"] = f.B.numpy()
            fac_arrays[f"lora_{li}_{nm}_scale"] = np.float32(f.scale)
        alayers[li] = lora_layer(li, **kw)
    adelta = lora_delta(source=WeightVersion(id="base"), target=WeightVersion(id="lora", parent_id="base", kind="lora"),
                        layers=alayers)
    fake = _types.SimpleNamespace(model=amodel, config=_types.SimpleNamespace(hidden_stride=2, propagator_rank=8))
    with torch.no_grad():
        apatches = DeltaKVEngine._analytic_patches(fake, ahidden, adelta)
        # the module functions on layer 1 with a seeded dx
        blk = amodel.blocks[1]
        adx = 0.05 * torch.randn(48, acfg.d_model, generator=ga)
        rn_y, rn_dy = rmsnorm_first_order(ahidden.h[1], adx, blk.attn_norm.weight, acfg.rms_eps)
        causal = torch.triu(torch.full((1, 48, 48), float("-inf")), diagonal=1)
        at_dh, at_dk, at_dv, _ = attention_first_order(
            rn_y, rn_dy, blk.q_proj.weight, blk.k_proj.weight, blk.v_proj.weight, blk.o_proj.weight, alayers[1],
            n_heads=acfg.n_heads, n_kv_heads=acfg.n_kv_heads, head_dim=acfg.head_dim, rope=amodel.rope,
            causal_mask=causal)
        mm_y, mm_dy = rmsnorm_first_order(ahidden.h_mid[1], adx, blk.mlp_norm.weight, acfg.rms_eps)
        ml_out = mlp_first_order(mm_y, mm_dy, blk.gate_proj.weight, blk.up_proj.weight, blk.down_proj.weight,
                                 alayers[1])
    np.savez_compressed(
        OUT / "analytic.npz",
        n_layers=np.int32(acfg.n_layers), d_model=np.int32(acfg.d_model), n_heads=np.int32(acfg.n_heads),
        n_kv=np.int32(acfg.n_kv_heads), hd=np.int32(acfg.head_dim), d_ff=np.int32(acfg.d_ff),
        eps=np.float32(acfg.rms_eps), rope_base=np.float32(acfg.rope_base), rope_max=np.int32(amodel.rope.max_seq),
        hidden_stride=np.int32(2), propagator_rank=np.int32(8),
        h=np.stack([t.numpy() for t in ahidden.h]), h_mid=np.stack([t.numpy() for t in ahidden.h_mid]),
        dk=np.stack([apatches[l].k_dense.numpy() for l in range(acfg.n_layers)]),
        dv=np.stack([apatches[l].v_dense.numpy() for l in range(acfg.n_layers)]),
        dx1=adx.numpy(), rn_y=rn_y.numpy(), rn_dy=rn_dy.numpy(), at_dh=at_dh.numpy(), at_dk=at_dk.numpy(),
        at_dv=at_dv.numpy(), ml_out=ml_out.numpy(),
        **fac_arrays,
        **{f"w_{k.replace('.', '_')}": v.detach().numpy() for k, v in amodel.state_dict().items()},
    )

    # ---------------------------------------------------------------- compare
    from deltakv.metrics import compare_kv

    rep = compare_kv(RefKV(k=pk, v=pv, version=WeightVersion(id="p")), RefKV(k=fk, v=fv, version=WeightVersion(id="f")))
    np.savez_compressed(
        OUT / "compare.npz", pk=pk.numpy(), pv=pv.numpy(), fk=fk.numpy(), fv=fv.numpy(),
        per_layer=np.array([[x.relative_l2_k, x.relative_l2_v, x.cosine_k, x.cosine_v] for x in rep.layers], np.float64),
        max_rel=np.float64(rep.max_relative_l2), mean_rel=np.float64(rep.mean_relative_l2),
        min_cos=np.float64(rep.min_cosine))

    # ------------------------------------------------------------------ probe
    from deltakv.patches.probe import apply_probe_to_cache, residual_gate, select_probes, weight_axis_scores
    from deltakv.patches.tensors import KVCache as RefKVCache
    from deltakv.patches.tensors import LowRankKVPatch as RefPatch

    gp = torch.Generator().manual_seed(9)
    n, dm, n_kv, hd, r = 96, 64, 2, 32, 4
    d_kv = n_kv * hd
    x_norm = torch.randn(n, dm, generator=gp)
    fk = LowRankFactors(A=torch.randn(r, dm, generator=gp) / dm ** 0.5, B=torch.randn(d_kv, r, generator=gp),
                        scale=0.5, name="k_proj")
    fv = LowRankFactors(A=torch.randn(r, dm, generator=gp) / dm ** 0.5, B=torch.randn(d_kv, r, generator=gp),
                        scale=0.25, name="v_proj")
    pdelta = lora_delta(source=WeightVersion(id="base"), target=WeightVersion(id="lora", parent_id="base", kind="lora"),
                        layers={0: lora_layer(0, k=fk, v=fv), 1: lora_layer(1, k=fk, v=fv)})
    scores = weight_axis_scores(x_norm, pdelta, 0)
    probes = select_probes(scores, 0.15, 4, 0.5)
    base_k = torch.randn(2, n, n_kv, hd, generator=gp)
    base_v = torch.randn(2, n, n_kv, hd, generator=gp)
    fresh = {}
    for l in range(2):
        ck = torch.randn(n, r, generator=gp) * 0.2
        cv = torch.randn(n, r, generator=gp) * 0.2
        noise = torch.randn(n, n_kv, hd, generator=gp) * 0.02
        outl = torch.zeros(n)
        outl[torch.randperm(n, generator=gp)[:6]] = 1.0  # a few tokens with a large unexplained residual
        fk_l = base_k[l] + (ck @ fk.B.T).view(n, n_kv, hd) + noise * (1 + 20 * outl.view(n, 1, 1))
        fv_l = base_v[l] + (cv @ fv.B.T).view(n, n_kv, hd) + noise
        fresh[l] = (fk_l, fv_l)
    kvp = RefKVCache(k=base_k.clone(), v=base_v.clone(), version=WeightVersion(id="base"))
    out_kv, ppatches, extra = apply_probe_to_cache(kvp, fresh, probes, 0.15, 0.40, layer_deltas=pdelta.layers,
                                                   subspace_rank=4, probe_layers={0})
    k_c0 = out_kv.k[0].clone()
    gate = residual_gate(base_k[0], k_c0, fresh[0][0], probes, 0.15, 0.40)
    np.savez_compressed(
        OUT / "probe.npz", x_norm=x_norm.numpy(), a_k=fk.A.numpy(), b_k=fk.B.numpy(), s_k=np.float32(fk.scale),
        a_v=fv.A.numpy(), b_v=fv.B.numpy(), s_v=np.float32(fv.scale), scores=scores.numpy(),
        probes=probes.numpy(), base_k=base_k.numpy(), base_v=base_v.numpy(),
        fresh_k=np.stack([fresh[l][0].numpy() for l in range(2)]), fresh_v=np.stack([fresh[l][1].numpy() for l in range(2)]),
        out_k=out_kv.k.numpy(), out_v=out_kv.v.numpy(), extra=extra.numpy(), gate=gate.numpy(),
        patch_k0=ppatches[0].k_dense.numpy(),
    )

    # ----------------------------------------------------------------- replay
    gr = torch.Generator().manual_seed(10)
    rb_k = torch.randn(3, 40, 2, 16, generator=gr)
    rb_v = torch.randn(3, 40, 2, 16, generator=gr)
    st1 = {0: RefPatch(layer_idx=0, k_codes=torch.randn(40, 3, generator=gr), k_basis=torch.randn(32, 3, generator=gr),
                       v_codes=torch.randn(40, 5, generator=gr), v_basis=torch.randn(32, 5, generator=gr)),
           2: RefPatch(layer_idx=2, k_codes=None, k_basis=None, v_codes=None, v_basis=None,
                       k_dense=torch.randn(40, 2, 16, generator=gr) * 0.1, v_dense=torch.randn(40, 2, 16, generator=gr) * 0.1)}
    st2 = {0: RefPatch(layer_idx=0, k_codes=None, k_basis=None, v_codes=None, v_basis=None,
                       k_dense=torch.randn(40, 2, 16, generator=gr) * 0.1, v_dense=torch.randn(40, 2, 16, generator=gr) * 0.1),
           1: RefPatch(layer_idx=1, k_codes=torch.randn(40, 2, generator=gr), k_basis=torch.randn(32, 2, generator=gr),
                       v_codes=torch.randn(40, 2, generator=gr), v_basis=torch.randn(32, 2, generator=gr))}
    rkv = RefKVCache(k=rb_k.clone(), v=rb_v.clone(), version=WeightVersion(id="base"))
    for stage in (st1, st2):  # the loop of engine._replay
        rkv = apply_layer_patches(rkv, stage)
    rep = {"base_k": rb_k.numpy(), "base_v": rb_v.numpy(), "out_k": rkv.k.numpy(), "out_v": rkv.v.numpy()}
    for si, stage in enumerate((st1, st2)):
        for l, ptc in stage.items():
            for nm in ("k_codes", "k_basis", "v_codes", "v_basis", "k_dense", "v_dense"):
                t = getattr(ptc, nm)
                if t is not None:
                    rep[f"s{si}_l{l}_{nm}"] = t.numpy()
    np.savez_compressed(OUT / "replay.npz", **rep)

    # ------------------------------------------------------------------- kivi
    from deltakv.metrics import _minmax_quantize, kivi_noise_floor
    from deltakv.patches.tensors import KVCache

    gk = torch.Generator().manual_seed(6)
    xv = torch.randn(70, 4, 64, generator=gk)            # [tokens, heads, dim]: groups along dim
    xk = torch.randn(96, 2, 64, generator=gk) * 0.5 + 0.1
    kq = _minmax_quantize(xk.reshape(96, -1).T.contiguous(), 4, 32).T.contiguous()  # groups along tokens
    kvc = KVCache(k=torch.randn(2, 64, 2, 32, generator=gk), v=torch.randn(2, 64, 2, 32, generator=gk),
                  version=WeightVersion(id="base"))
    np.savez_compressed(OUT / "kivi.npz", xv=xv.numpy(), xv_q=_minmax_quantize(xv, 4, 32).numpy(),
                        xk=xk.numpy(), xk_q=kq.numpy(), floor_k=kvc.k.numpy(), floor_v=kvc.v.numpy(),
                        floor=np.float64(kivi_noise_floor(kvc, bits=4, group_size=32)))


def _state_from_oracle(model, w: dict) -> None:
    """Load oracle-named numpy weights into a reference ToyTransformer."""
    import torch

    sd = model.state_dict()
    for key in sd:
        name = key.replace(".", "_")
        if name == "lm_head_weight" and name not in w:
            name = "embed_weight"
        sd[key] = torch.from_numpy(np.ascontiguousarray(w[name]))
    model.load_state_dict(sd)


def smol_kl_case(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    sys.path.insert(0, str(OUT.parent.parent))
    import torch

    from deltakv.deltas.descriptor import lora_layer
    from deltakv.deltas.factors import LowRankFactors
    from deltakv.deltas.lora import lora_delta
    from deltakv.metrics import next_token_kl
    from deltakv.model import ToyConfig, ToyTransformer
    from deltakv.patches.compose import apply_layer_patches
    from deltakv.patches.exact import zeroth_order_patches
    from deltakv.types import WeightVersion
    from tests import _smol_model as SM

    torch.set_num_threads(8)
    torch.set_grad_enabled(False)
    cfg = ToyConfig(vocab_size=SM.VOCAB, d_model=SM.D, n_layers=SM.N_LAYERS, n_heads=SM.N_HEADS, n_kv_heads=SM.N_KV,
                    d_ff=SM.D_FF, max_seq=SM.SEQ, rms_eps=SM.EPS, rope_base=SM.ROPE_BASE)
    model = ToyTransformer(cfg)
    w = SM.weights()
    _state_from_oracle(model, w)
    tokens = torch.from_numpy(SM.tokens())
    _, kv_base, hidden = model.prefill(tokens)
    dl = SM.delta(w)
    layers = {i: lora_layer(i, **{name[0]: LowRankFactors(A=torch.from_numpy(A), B=torch.from_numpy(B), scale=s,
                                                          name=name)
                                  for name, (A, B, s) in projs.items()})
              for i, projs in dl.items()}
    delta = lora_delta(source=WeightVersion(id="base"), target=WeightVersion(id="lora", parent_id="base", kind="lora"),
                       layers=layers)
    xn = model.rmsnorm_tensors(hidden)
    patches = zeroth_order_patches(xn, delta, n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, rope=model.rope)
    patched = apply_layer_patches(kv_base, patches)
    stale_logits = model.logits_from_kv(tokens, kv_base)
    model.apply_delta(delta, version=WeightVersion(id="lora"))
    fresh_logits, kv_fresh, _ = model.prefill(tokens)
    patched_logits = model.logits_from_kv(tokens, patched)
    h = torch.stack(list(hidden.h))
    norms = lambda t: np.array([float(t[l].double().norm()) for l in range(t.shape[0])])
    np.savez_compressed(
        OUT / "smol_kl.npz",
        tokens=tokens.numpy(), fresh_logits=fresh_logits[-1].numpy(), patched_logits=patched_logits.numpy(),
        kl_ref=np.float64(next_token_kl(fresh_logits[-1], patched_logits)),
        kl_stale=np.float64(next_token_kl(fresh_logits[-1], stale_logits)),
        h_head=h[:, :4].numpy(), h_tail=h[:, -4:].numpy(), h_norms=norms(h),
        k_tail=kv_base.k[:, -4:].numpy(), v_tail=kv_base.v[:, -4:].numpy(),
        k_norms=norms(kv_base.k), v_norms=norms(kv_base.v),
        patched_k_norms=norms(patched.k), patched_v_norms=norms(patched.v),
        fresh_k_norms=norms(kv_fresh.k), fresh_v_norms=norms(kv_fresh.v),
    )


def engine_case(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    import copy

    import torch

    import deltakv.engine as E
    from deltakv.config import DeltaKVConfig
    from deltakv.connectors.vllm import DeltaKVConnector
    from deltakv.deltas.descriptor import lora_layer
    from deltakv.deltas.factors import random_lora_factors
    from deltakv.deltas.lora import lora_delta
    from deltakv.model import ToyConfig, ToyTransformer
    from deltakv.types import CompatibilityLevel, WeightVersion

    torch.set_num_threads(4)
    torch.set_grad_enabled(False)
    cfg = ToyConfig(n_layers=4, d_model=64, n_heads=4, n_kv_heads=2, d_ff=128, vocab_size=256)
    torch.manual_seed(0)
    model0 = ToyTransformer(cfg)
    state0 = copy.deepcopy(model0.state_dict())
    tokens = torch.randint(0, 256, (64,), generator=torch.Generator().manual_seed(0))
    rng = torch.Generator().manual_seed(1)
    d_kv, d_q = cfg.n_kv_heads * cfg.head_dim, cfg.n_heads * cfg.head_dim
    layers, fac = {}, {}
    for i in range(cfg.n_layers):
        k = random_lora_factors(cfg.d_model, d_kv, 4, scale=0.01, generator=rng, name="k_proj")
        v = random_lora_factors(cfg.d_model, d_kv, 4, scale=0.01, generator=rng, name="v_proj")
        q = random_lora_factors(cfg.d_model, d_q, 4, scale=0.01, generator=rng, name="q_proj")
        layers[i] = lora_layer(i, k=k, v=v, q=q)
        for n_, f in (("k", k), ("v", v), ("q", q)):
            fac.setdefault(f"a_{n_}", []).append(f.A.numpy())
            fac.setdefault(f"b_{n_}", []).append(f.B.numpy())
            fac.setdefault(f"s_{n_}", []).append(float(f.scale))
    delta = lora_delta(source=WeightVersion(id="base"), target=WeightVersion(id="lora-v1", parent_id="base",
                                                                              kind="lora"), layers=layers)
    out = {k: np.stack(v) if k[0] in "ab" else np.array(v, np.float32) for k, v in fac.items()}
    out["tokens"] = tokens.numpy()
    names = ("zeroth_order_patches", "weight_axis_scores", "select_probes", "apply_probe_to_cache")
    orig = {n: getattr(E, n) for n in names}
    for route, request, gate_off in (("exact", "exact", False), ("hybrid", "hybrid", False),
                                     ("subspace", "probe", True)):
        rec = {}

        def zeroth(xn, d, **kw):
            rec["xn"] = np.stack([xn[l].numpy() for l in sorted(xn)])
            return orig["zeroth_order_patches"](xn, d, **kw)

        def scores(x, d, layer_idx=0):
            rec["score_x"], rec["score_layer"] = x.numpy().copy(), np.int32(layer_idx)
            r = orig["weight_axis_scores"](x, d, layer_idx)
            rec["scores"] = r.numpy().copy()
            return r

        def select(sc, ratio, mn=4, mx=0.5):
            rec["ratio"], rec["min_tokens"], rec["max_ratio"] = np.float64(ratio), np.int32(mn), np.float64(mx)
            r = orig["select_probes"](sc, ratio, mn, mx)
            rec["probes"] = r.numpy().copy()
            return r

        def probe(kv, fresh, probes, thr=0.15, maxr=0.40, *, layer_deltas=None, subspace_rank=8,
                  probe_layers=None, skip_layers=None):
            if gate_off:
                probe_layers = set()
            rec["kv_in_k"], rec["kv_in_v"] = kv.k.numpy().copy(), kv.v.numpy().copy()
            ls = sorted(fresh)
            rec["fresh_layers"] = np.array(ls, np.int32)
            rec["fresh_k"] = np.stack([fresh[l][0].numpy() for l in ls])
            rec["fresh_v"] = np.stack([fresh[l][1].numpy() for l in ls])
            rec["thr"], rec["maxr"], rec["subspace_rank"] = np.float64(thr), np.float64(maxr), np.int32(subspace_rank)
            enc = lambda s_: np.array([-1], np.int32) if s_ is None else np.array(sorted(s_), np.int32)
            rec["probe_layers"], rec["skip_layers"] = enc(probe_layers), enc(skip_layers)
            res = orig["apply_probe_to_cache"](kv, fresh, probes, thr, maxr, layer_deltas=layer_deltas,
                                               subspace_rank=subspace_rank, probe_layers=probe_layers,
                                               skip_layers=skip_layers)
            rec["kv_out_k"], rec["kv_out_v"], rec["extra"] = res[0].k.numpy().copy(), res[0].v.numpy().copy(), \
                res[2].numpy().copy()
            return res

        model = ToyTransformer(cfg)
        model.load_state_dict(state0)
        eng = E.DeltaKVEngine(model, DeltaKVConfig())
        eng.prefill(tokens)
        entry = next(iter(eng.store.items()))
        base_k, base_v = entry.base.k.numpy().copy(), entry.base.v.numpy().copy()
        eng.commit_delta(delta)
        for n_, fn in zip(names, (zeroth, scores, select, probe)):
            setattr(E, n_, fn)
        try:
            res = eng.evaluate_against_fresh(tokens, route=request)
        finally:
            for n_ in names:
                setattr(E, n_, orig[n_])
        assert res.decision.level is CompatibilityLevel.PATCHED, res.decision
        _, fresh_kv, _ = model.prefill(tokens)
        out[f"{route}_base_k"], out[f"{route}_base_v"] = base_k, base_v
        out[f"{route}_k"], out[f"{route}_v"] = res.kv.k.numpy(), res.kv.v.numpy()
        out[f"{route}_kl"] = np.float64(res.report.next_token_kl)
        out[f"{route}_max_rel_l2"] = np.float64(res.report.max_relative_l2)
        out[f"{route}_decision_route"] = np.array(res.decision.route.value)
        for k, v in rec.items():
            out[f"{route}_{k}"] = v
        if route == "exact":
            out["fresh_k"], out["fresh_v"] = fresh_kv.k.numpy(), fresh_kv.v.numpy()
            sd = model.state_dict()
            for key, t in sd.items():
                out["w_" + key.replace(".", "_")] = t.numpy().copy()
            out["rope_cos"] = model.rope.cos_cached[:, : cfg.head_dim // 2].numpy()
            out["rope_sin"] = model.rope.sin_cached[:, : cfg.head_dim // 2].numpy()
            # the connector writes the materialised view into vLLM's paged buffers
            bs, nb = 16, 9
            gp = torch.Generator().manual_seed(3)
            table = torch.randperm(nb, generator=gp)[:4].tolist()
            kc = [torch.randn(nb, bs, cfg.n_kv_heads, cfg.head_dim, generator=gp).to(torch.bfloat16)
                  for _ in range(cfg.n_layers)]
            vc = [torch.randn(nb, bs, cfg.n_kv_heads, cfg.head_dim, generator=gp).to(torch.bfloat16)
                  for _ in range(cfg.n_layers)]
            out["conn_k_in"] = np.stack([bf16_bits(c) for c in kc])
            out["conn_v_in"] = np.stack([bf16_bits(c) for c in vc])
            # unbound: with vLLM 0.22 installed the connector's constructor fails (it assigns the
            # base class's read-only `role` property); patch_paged itself does not use `self`
            DeltaKVConnector.patch_paged(None, res.kv, kc, vc, table, bs)
            out["conn_k_out"] = np.stack([bf16_bits(c) for c in kc])
            out["conn_v_out"] = np.stack([bf16_bits(c) for c in vc])
            out["conn_table"] = np.array(table, np.int32)
            out["conn_bs"] = np.int32(bs)
    for key in ("n_heads", "n_kv_heads", "head_dim", "n_layers"):
        out[key] = np.int32(getattr(cfg, key))
    out["eps"] = np.float32(cfg.rms_eps)
    np.savez_compressed(OUT / "engine.npz", **out)


def smol_dense_case(ref_src: str) -> None:
    """smol_dense.npz: a full-rank dW on k/v of every layer of the SmolLM2-shaped stack through
    the reference's exact route as LowRankFactors(A=dW, B=I, scale=1) (rmsnorm_tensors ->
    zeroth_order_patches -> apply_layer_patches), then apply_delta and a fresh prefill."""
    sys.path.insert(0, ref_src)
    sys.path.insert(0, str(OUT.parent.parent))
    import torch

    from deltakv.deltas.descriptor import lora_layer
    from deltakv.deltas.factors import LowRankFactors
    from deltakv.deltas.lora import lora_delta
    from deltakv.metrics import next_token_kl
    from deltakv.model import ToyConfig, ToyTransformer
    from deltakv.patches.compose import apply_layer_patches
    from deltakv.patches.exact import zeroth_order_patches
    from deltakv.types import WeightVersion
    from tests import _smol_model as SM

    torch.set_num_threads(8)
    torch.set_grad_enabled(False)
    cfg = ToyConfig(vocab_size=SM.VOCAB, d_model=SM.D, n_layers=SM.N_LAYERS, n_heads=SM.N_HEADS, n_kv_heads=SM.N_KV,
                    d_ff=SM.D_FF, max_seq=SM.SEQ, rms_eps=SM.EPS, rope_base=SM.ROPE_BASE)
    model = ToyTransformer(cfg)
    w = SM.weights()
    _state_from_oracle(model, w)
    tokens = torch.from_numpy(SM.tokens())
    _, kv_base, hidden = model.prefill(tokens)
    dd = SM.dense_delta(w)
    d_kv = SM.N_KV * SM.HD
    eye = torch.eye(d_kv)
    layers = {i: lora_layer(i, k=LowRankFactors(A=torch.from_numpy(p["k_proj"]), B=eye, scale=1.0, name="k_proj"),
                            v=LowRankFactors(A=torch.from_numpy(p["v_proj"]), B=eye, scale=1.0, name="v_proj"))
              for i, p in dd.items()}
    delta = lora_delta(source=WeightVersion(id="base"), target=WeightVersion(id="rl", parent_id="base", kind="rl_step"),
                       layers=layers)
    xn = model.rmsnorm_tensors(hidden)
    patches = zeroth_order_patches(xn, delta, n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, rope=model.rope)
    patched = apply_layer_patches(kv_base, patches)
    stale_logits = model.logits_from_kv(tokens, kv_base)
    model.apply_delta(delta, version=WeightVersion(id="rl"))
    fresh_logits, _, _ = model.prefill(tokens)
    patched_logits = model.logits_from_kv(tokens, patched)
    np.savez_compressed(OUT / "smol_dense.npz", tokens=tokens.numpy(), fresh_logits=fresh_logits[-1].numpy(),
                        patched_logits=patched_logits.numpy(), stale_logits=stale_logits.numpy(),
                        kl_ref=np.float64(next_token_kl(fresh_logits[-1], patched_logits)),
                        kl_stale=np.float64(next_token_kl(fresh_logits[-1], stale_logits)))


CASES = {"core": core_cases, "engine": engine_case, "smol_kl": smol_kl_case, "smol_dense": smol_dense_case}


def main(ref_src: str, cases=None) -> None:
    for name in cases or list(CASES):
        CASES[name](ref_src)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference checkout>/src [core|engine|smol_kl|smol_dense ...]")
    main(sys.argv[1], sys.argv[2:] or None)
