"""Next-token KL of the patched cache beyond the 4-layer toy: the SmolLM2-135M shape, for the
exact route (below), the int4 subspace route and the dense-dW route (their own docstrings).

Weights, tokens and the rank-8 q/k/v/o LoRA come from seeds (tests/_smol_model.py: d=576,
9 / 3 heads of 64, SwiGLU 1536, vocab 49152, 2048 tokens; 4 of the 30 layers so the fp32
oracle prefill stays within a test's time).  The oracle prefill gives the stored layer
inputs and the stale K/V (pinned against the reference's own run by
tests/test_oracle_golden.py::test_smol_prefill_and_kl_golden).  This build then patches the
way the throughput run does: layer inputs stored as f16 codes with power-of-two row scales
and per-row sums of squared codes, RMSNorm folded, rank-8 k/v factors, RoPE, bf16 paged K/V
through a permuted block table, one fused launch.  The patched pages are scored by the
oracle's last-token pass under the updated weights.

Bars (src/deltakv/metrics.py:92-98): KL(fresh || patched) within 1e-4 nats of the
reference's KL(fresh || patched_reference); and, tighter, KL(patched_reference || patched)
below 1e-6 nats — 25x what storing the reference's own patched cache in bf16 costs (4e-8),
while the unpatched cache sits 6.5e-5 from fresh.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deltakv_b200 as dkv
from deltakv_b200 import ops
from oracle import exact as OX
from oracle import model as OM
from tests import _smol_model as SM
from tests.conftest import golden
from tests.helpers import bits_from_bf16

pytestmark = pytest.mark.gpu


def test_smollm2_shape_next_token_kl(cuda):
    g = golden("smol_kl")
    w = SM.weights()
    dl = SM.delta(w)
    toks = g["tokens"]
    tabs = OX.rope_tables(SM.HD, SM.SEQ, SM.ROPE_BASE)
    kw = dict(n_layers=SM.N_LAYERS, n_heads=SM.N_HEADS, n_kv=SM.N_KV, hd=SM.HD, eps=SM.EPS, rope=tabs)
    _, k0, v0, h = OM.prefill(w, toks, **kw)
    L_, n = SM.N_LAYERS, SM.SEQ
    # stored activations as the engine would keep them: f16 codes, row scale, sums of squares
    xq, xs, ssq = dkv.quantize_rows(torch.from_numpy(h).to(cuda), torch.float16, with_sumsq=True)
    # the stale cache in bf16 pages through a permuted block table
    bs = 16
    nblk = n // bs
    perm = np.random.default_rng(9).permutation(nblk + 3)[:nblk].astype(np.int32)
    pages = []
    for src in (k0, v0):
        p = torch.randn(L_, nblk + 3, bs, SM.N_KV, SM.HD, generator=torch.Generator().manual_seed(4))
        p[:, torch.from_numpy(perm).long()] = torch.from_numpy(src).view(L_, nblk, bs, SM.N_KV, SM.HD)
        pages.append(p.to(torch.bfloat16).to(cuda))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    patcher = dkv.ExactPatcher(SM.D, SM.N_KV, SM.HD, rank_k=SM.RANK, rank_v=SM.RANK, x_dtype=torch.float16,
                               rope=(torch.from_numpy(tabs[0]), torch.from_numpy(tabs[1])), norm_eps=SM.EPS)
    fac = lambda p, i: np.stack([dl[l][p][i] for l in range(L_)])
    scaled_b = lambda p: np.stack([dl[l][p][1] * dl[l][p][2] for l in range(L_)])
    packed = patcher.pack(t(fac("k_proj", 0)), t(scaled_b("k_proj")), t(fac("v_proj", 0)), t(scaled_b("v_proj")),
                          1.0, 1.0, norm_weight=t(np.stack([w[f"blocks_{l}_attn_norm_weight"] for l in range(L_)])))
    seqs = ops.SeqBatchTensors(cu_seqlens=torch.tensor([0, n], dtype=torch.int32, device=cuda),
                               block_tables=t(perm[None]), max_seq_len=n)
    patcher.apply(xq, packed, [pages[0][l] for l in range(L_)], [pages[1][l] for l in range(L_)], seqs,
                  x_scale=xs, apply_norm=True, x_sumsq=ssq, check=True)
    torch.cuda.synchronize()
    got = []
    for p in pages:
        bits = bits_from_bf16(p)
        f = (bits.astype(np.uint32) << 16).view(np.float32).reshape(p.shape)
        got.append(f[:, perm].reshape(L_, n, SM.N_KV, SM.HD))
    logits = OM.logits_from_kv(SM.merged(w, dl), toks, got[0], got[1], **kw)
    kl = OM.next_token_kl(g["fresh_logits"], logits)
    assert abs(kl - float(g["kl_ref"])) < 1e-4, (kl, float(g["kl_ref"]))
    assert OM.next_token_kl(g["patched_logits"], logits) < 1e-6
    # the patch moved the cache: the stale cache is measurably further from fresh
    stale = OM.logits_from_kv(SM.merged(w, dl), toks, k0, v0, **kw)
    assert OM.next_token_kl(g["patched_logits"], stale) > 10 * OM.next_token_kl(g["patched_logits"], logits)


def test_smollm2_shape_int4_subspace_route_kl(cuda):
    """The multi-adapter maintenance route on a real stack: the stale cache of the SmolLM2-shaped
    decoder (4 layers, 2048 tokens, d_kv 192) stored KIVI int4, corrected per layer toward the
    fresh prefill under the LoRA'd weights from every 10th token (K basis: the probe residual's
    top-8 subspace; V basis: the adapter's LoRA B), stored int4 again; scored by next-token KL
    against the fresh logits.  Held to the oracle composition (KIVI dequantise ->
    subspace_correct -> quantise, fp32): KL within 1e-4 nats of the oracle's, and the two
    corrected caches' next-token distributions within 1e-6 nats of each other."""
    from deltakv_b200 import kivi as K
    from oracle import kivi as OK
    from oracle import subspace as OS

    g = golden("smol_kl")
    w = SM.weights()
    dl = SM.delta(w)
    w1 = SM.merged(w, dl)
    toks = g["tokens"]
    tabs = OX.rope_tables(SM.HD, SM.SEQ, SM.ROPE_BASE)
    kw = dict(n_layers=SM.N_LAYERS, n_heads=SM.N_HEADS, n_kv=SM.N_KV, hd=SM.HD, eps=SM.EPS, rope=tabs)
    _, k0, v0, _ = OM.prefill(w, toks, **kw)
    _, k1, v1, _ = OM.prefill(w1, toks, **kw)
    L_, n, d = SM.N_LAYERS, SM.SEQ, SM.N_KV * SM.HD
    probes = np.arange(0, n, 10)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    ours, ref = {"k": [], "v": []}, {"k": [], "v": []}
    probs = []
    for l in range(L_):
        for mode, stale, fresh in (("k", k0[l], k1[l]), ("v", v0[l], v1[l])):
            c, s, z = OK.quantize(stale.reshape(n, d), mode)
            basis = dl[l]["v_proj"][1] if mode == "v" else None  # the adapter's LoRA B [d_kv, r]
            reused = OK.dequantize(c, s, z, mode)
            corr, _, _ = OS.subspace_correct(reused.reshape(n, SM.N_KV, SM.HD), fresh, probes, basis=basis,
                                             rank=SM.RANK)
            ref[mode].append(OK.dequantize(*OK.quantize(corr.reshape(n, d), mode), mode).reshape(n, SM.N_KV, SM.HD))
            probs.append(K.SubspaceProblem(base=K.KiviTensor(t(c), t(s), t(z), mode), fresh=t(fresh.reshape(n, d)),
                                           probe_index=t(probes), basis=None if basis is None else t(basis),
                                           rank=SM.RANK, out=K.KiviTensor.empty(n, d, mode, cuda)))
    K.subspace_correct(probs)
    torch.cuda.synchronize()
    for i, pb in enumerate(probs):
        mode = "k" if i % 2 == 0 else "v"
        ours[mode].append(K.dequantize(pb.out).cpu().numpy().reshape(n, SM.N_KV, SM.HD))
    stack = lambda m: np.stack(m)
    lo = OM.logits_from_kv(w1, toks, stack(ours["k"]), stack(ours["v"]), **kw)
    lr = OM.logits_from_kv(w1, toks, stack(ref["k"]), stack(ref["v"]), **kw)
    kl_ours = OM.next_token_kl(g["fresh_logits"], lo)
    kl_ref = OM.next_token_kl(g["fresh_logits"], lr)
    stale = [OK.dequantize(*OK.quantize(x[l].reshape(n, d), m), m).reshape(n, SM.N_KV, SM.HD)
             for x, m in ((k0, "k"), (v0, "v")) for l in range(L_)]
    kl_stale = OM.next_token_kl(g["fresh_logits"], OM.logits_from_kv(w1, toks, np.stack(stale[:L_]),
                                                                      np.stack(stale[L_:]), **kw))
    print("int4 route KL: ours", kl_ours, "oracle", kl_ref, "stale int4", kl_stale,
          "ours vs oracle", OM.next_token_kl(lr, lo))
    assert abs(kl_ours - kl_ref) < 1e-4
    assert OM.next_token_kl(lr, lo) < 1e-6
    assert kl_ours < kl_stale  # the correction moved the int4 cache toward fresh


def test_smollm2_shape_dense_route_kl(cuda):
    """The RL-step route on the same stack (reduced depth; the Llama-3-70B stack itself has no
    fp32 oracle that fits): a full-rank dW on k/v of every layer (relative norm 0.02, bf16
    values), stored layer inputs in bf16 with the RMSNorm weight folded into the packed dW and
    the per-row 1/rms computed from them, one tensor-core GEMM launch into bf16 pages.  Against
    the reference's exact route with A=dW, B=I (tests/golden/smol_dense.npz): KL(fresh ||
    patched) within 1e-4 nats of the reference's, KL(patched_reference || patched) below 1e-6
    (bf16 storage of X and of the pages alone costs 3.5e-8)."""
    g = golden("smol_dense")
    w = SM.weights()
    dd = SM.dense_delta(w)
    w1 = SM.merged_dense(w, dd)
    toks = g["tokens"]
    tabs = OX.rope_tables(SM.HD, SM.SEQ, SM.ROPE_BASE)
    kw = dict(n_layers=SM.N_LAYERS, n_heads=SM.N_HEADS, n_kv=SM.N_KV, hd=SM.HD, eps=SM.EPS, rope=tabs)
    _, k0, v0, h = OM.prefill(w, toks, **kw)
    L_, n = SM.N_LAYERS, SM.SEQ
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    x = t(h).to(torch.bfloat16)
    bs = 16
    nblk = n // bs
    perm = np.random.default_rng(11).permutation(nblk + 2)[:nblk].astype(np.int32)
    pages = []
    for src in (k0, v0):
        p = torch.randn(L_, nblk + 2, bs, SM.N_KV, SM.HD, generator=torch.Generator().manual_seed(6))
        p[:, torch.from_numpy(perm).long()] = torch.from_numpy(src).view(L_, nblk, bs, SM.N_KV, SM.HD)
        pages.append(p.to(torch.bfloat16).to(cuda))
    patcher = dkv.DensePatcher(SM.D, SM.N_KV, SM.HD, rope=(torch.from_numpy(tabs[0]), torch.from_numpy(tabs[1])),
                               norm_eps=SM.EPS)
    packed = patcher.pack(t(np.stack([dd[l]["k_proj"] for l in range(L_)])),
                          t(np.stack([dd[l]["v_proj"] for l in range(L_)])),
                          norm_weight=t(np.stack([w[f"blocks_{l}_attn_norm_weight"] for l in range(L_)])))
    seqs = ops.SeqBatchTensors(cu_seqlens=torch.tensor([0, n], dtype=torch.int32, device=cuda),
                               block_tables=t(perm[None]), max_seq_len=n)
    patcher.apply(x, packed, [pages[0][l] for l in range(L_)], [pages[1][l] for l in range(L_)], seqs,
                  x_scale=patcher.norm_scale(x), check=True)
    torch.cuda.synchronize()
    got = []
    for p in pages:
        f = (bits_from_bf16(p).astype(np.uint32) << 16).view(np.float32).reshape(p.shape)
        got.append(f[:, perm].reshape(L_, n, SM.N_KV, SM.HD))
    logits = OM.logits_from_kv(w1, toks, got[0], got[1], **kw)
    kl = OM.next_token_kl(g["fresh_logits"], logits)
    assert abs(kl - float(g["kl_ref"])) < 1e-4, (kl, float(g["kl_ref"]))
    assert OM.next_token_kl(g["patched_logits"], logits) < 1e-6
    stale = OM.next_token_kl(g["patched_logits"], g["stale_logits"])
    assert stale > 10 * OM.next_token_kl(g["patched_logits"], logits)
