"""Parity at the geometries the throughput figures are quoted on, through the C ABI.

* Llama-3-8B shape (exact route): d=4096, 8 KV heads x 128, rank-16 k/v LoRA (the tcgen05
  kernel) and rank 64 (the mma.sync kernel), fp8-e4m3 stored activations with per-token
  absmax scales, RMSNorm with a non-unit weight (from the stored per-row sums of squared
  codes and from the tensor cores' X.X^T diagonal), RoPE theta 5e5, bf16 pages, block 16,
  permuted block table, 2 layers x 3 sequences of (4096, 1000, 17) tokens.
* SmolLM2-135M shape (exact route): d=576, 3 KV heads x 64, rank 8, f16 stored activations.
* Llama-3-70B shape (dense dW route): d=8192, 8 KV heads x 128, bf16 activations.

Oracle: the numpy restatement of the reference's exact branch (RMSNorm -> exact_kv_patch ->
materialize -> scatter_into_paged, src/deltakv/model.py:48-56, patches/exact.py:14-63,
patches/tensors.py:105-123, paged.py:8-43); the dense route as LowRankFactors(A=dW, B=I).

Tolerances: bf16 pages within rel-L2 1e-3 of the oracle's bf16 result, untouched slots
bit-identical and >= 99 % of touched elements bit-identical (at these shapes the patch is
~1.6 % of a page, so a delta off by 5 % would leave ~87 % equal); the delta itself, written
to fp32 pages (f16 for the dense route, which stores bf16/f16 only), within rel-L2 1e-3 of
the oracle's fp32 delta.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import deltakv_b200 as dkv
from deltakv_b200 import ops
from oracle import dense as OD
from oracle import exact as OX
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits
from tests.helpers import bf16_from_bits, bits_from_bf16, e4m3_from_bits, rel_l2

pytestmark = pytest.mark.gpu
REL_TOL = 1e-3
BIT_EQUAL_MIN = 0.99
LLAMA8B = dict(d=4096, n_kv=8, hd=128, theta=500000.0, xdt="e4m3", lens=(4096, 1000, 17))
SMOL = dict(d=576, n_kv=3, hd=64, theta=10000.0, xdt="f16", lens=(2048, 700, 5))


def _tables(rng, lens, bs):
    need = [(n + bs - 1) // bs for n in lens]
    nb = sum(need) + 5
    perm = rng.permutation(nb).astype(np.int32)
    tables = np.zeros((len(lens), max(need)), np.int32)
    k = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[k:k + n]
        k += n
    return tables, nb


def _touched(nb, tables, lens, bs):
    m = np.zeros(nb, bool)
    for b, n in enumerate(lens):
        m[tables[b, :(n + bs - 1) // bs]] = True
    return m


def _exact_case(geo, rank, seed, n_layers=2, bs=16):
    """Inputs as the throughput run makes them: residual-stream-like rows (N(0,1) times a
    per-token magnitude in [0.5, 1.5)), A ~ N(0, 1/d), B ~ N(0, 1), the LoRA scale set so
    ||s B A||_F = 1e-2 ||W||_F for W ~ N(0, 0.02^2)."""
    rng = np.random.default_rng(seed)
    d, n_kv, hd = geo["d"], geo["n_kv"], geo["hd"]
    d_kv = n_kv * hd
    lens = list(geo["lens"])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    rows = int(cu[-1])
    h = rng.standard_normal((n_layers, rows, d), dtype=np.float32)
    h *= (0.5 + rng.random((n_layers, rows, 1), dtype=np.float32))
    if geo["xdt"] == "e4m3":
        xs = (np.abs(h).max(-1) / 448.0).astype(np.float32)
        # torch's round-to-nearest-even e4m3 cast (fast); both sides then read the same bits
        xbits = torch.from_numpy(h / xs[..., None]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    else:  # f16 codes with a power-of-two row scale
        xs = np.exp2(np.ceil(np.log2(np.abs(h).max(-1) / 1024.0))).astype(np.float32)
        xbits = (h / xs[..., None]).astype(np.float16)
    codes = OX.dequant_x(xbits.reshape(-1, d), geo["xdt"], None).reshape(n_layers, rows, d)
    sumsq = (codes.astype(np.float64) ** 2).sum(-1).astype(np.float32)
    w_norm = 0.02 * math.sqrt(d_kv * d)
    fac = []
    for _ in range(n_layers):
        pair = []
        for _p in "kv":
            A = (rng.standard_normal((rank, d)) / math.sqrt(d)).astype(np.float32)
            B = rng.standard_normal((d_kv, rank)).astype(np.float32)
            s = float(1e-2 * w_norm / np.linalg.norm(B @ A))
            pair.append((A, B, s))
        fac.append(tuple(pair))
    norm_w = (1.0 + 0.05 * rng.standard_normal((n_layers, d))).astype(np.float32)
    tables, nb = _tables(rng, lens, bs)
    tabs = OX.rope_tables(hd, max(lens), geo["theta"])
    return dict(lens=lens, cu=cu, xbits=xbits, xs=xs, sumsq=sumsq, fac=fac, norm_w=norm_w, tables=tables, nb=nb,
                tabs=tabs, bs=bs, L=n_layers, rng=rng)


def _run_exact(cuda, geo, case, rank, k_pages, v_pages, *, sumsq: bool):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    xdtype = torch.float8_e4m3fn if geo["xdt"] == "e4m3" else torch.float16
    patcher = dkv.ExactPatcher(geo["d"], geo["n_kv"], geo["hd"], rank_k=rank, rank_v=rank, x_dtype=xdtype,
                               rope=(torch.from_numpy(case["tabs"][0]), torch.from_numpy(case["tabs"][1])),
                               norm_eps=1e-5)
    st = lambda i, j: t(np.stack([case["fac"][l][i][j] for l in range(case["L"])]))
    # per-layer LoRA scales folded into B (the packer takes one scale per projection)
    b_k = t(np.stack([case["fac"][l][0][1] * case["fac"][l][0][2] for l in range(case["L"])]))
    b_v = t(np.stack([case["fac"][l][1][1] * case["fac"][l][1][2] for l in range(case["L"])]))
    packed = patcher.pack(st(0, 0), b_k, st(1, 0), b_v, 1.0, 1.0, norm_weight=t(case["norm_w"]))
    x = e4m3_from_bits(case["xbits"], cuda) if geo["xdt"] == "e4m3" else t(case["xbits"])
    seqs = ops.SeqBatchTensors(cu_seqlens=t(case["cu"]), block_tables=t(case["tables"]),
                               max_seq_len=max(case["lens"]))
    patcher.apply(x, packed, k_pages, v_pages, seqs, x_scale=t(case["xs"]), apply_norm=True, check=True,
                  x_sumsq=t(case["sumsq"]) if sumsq else None)
    torch.cuda.synchronize()


def _oracle_exact(geo, case, k_pages, v_pages, kind):
    OX.exact_patch_paged(x=case["xbits"], x_dtype=geo["xdt"],
                         x_scale=case["xs"], norm_w=case["norm_w"], eps=1e-5, factors=case["fac"],
                         cu_seqlens=case["cu"], block_tables=case["tables"], k_pages=k_pages, v_pages=v_pages,
                         n_kv=geo["n_kv"], hd=geo["hd"], rope=case["tabs"], kind=kind)


@pytest.mark.parametrize("geo,rank", [(LLAMA8B, 16), (LLAMA8B, 64), (SMOL, 8)],
                         ids=["llama8b-r16", "llama8b-r64", "smollm2-r8"])
def test_exact_bf16_pages_at_bench_geometry(cuda, geo, rank):
    case = _exact_case(geo, rank, seed=11 + rank)
    L_, nb, bs, n_kv, hd = case["L"], case["nb"], case["bs"], geo["n_kv"], geo["hd"]
    base = [[f32_to_bf16_bits(case["rng"].standard_normal((nb, bs, n_kv, hd), dtype=np.float32)) for _ in range(L_)]
            for _kv in range(2)]
    kref = [b.copy() for b in base[0]]
    vref = [b.copy() for b in base[1]]
    _oracle_exact(geo, case, kref, vref, "bf16")
    touched = _touched(nb, case["tables"], case["lens"], bs)
    for sumsq in (True, False):
        kp = [bf16_from_bits(b, cuda) for b in base[0]]
        vp = [bf16_from_bits(b, cuda) for b in base[1]]
        _run_exact(cuda, geo, case, rank, kp, vp, sumsq=sumsq)
        for l in range(L_):
            for got_t, ref, inp in ((kp[l], kref[l], base[0][l]), (vp[l], vref[l], base[1][l])):
                got = bits_from_bf16(got_t)
                assert np.array_equal(got[~touched], inp[~touched])
                err = rel_l2(bf16_bits_to_f32(got[touched]), bf16_bits_to_f32(ref[touched]))
                assert err < REL_TOL, (sumsq, l, err)
                eq = (got[touched] == ref[touched]).mean()
                assert eq >= BIT_EQUAL_MIN, (sumsq, l, eq)


@pytest.mark.parametrize("geo,rank", [(LLAMA8B, 16), (LLAMA8B, 64), (SMOL, 8)],
                         ids=["llama8b-r16", "llama8b-r64", "smollm2-r8"])
def test_exact_delta_fp32_pages_at_bench_geometry(cuda, geo, rank):
    """The delta itself, accumulated into zeroed fp32 pages: no page rounding hides it."""
    case = _exact_case(geo, rank, seed=23 + rank)
    L_, nb, bs, n_kv, hd = case["L"], case["nb"], case["bs"], geo["n_kv"], geo["hd"]
    kref = [np.zeros((nb, bs, n_kv, hd), np.float32) for _ in range(L_)]
    vref = [np.zeros((nb, bs, n_kv, hd), np.float32) for _ in range(L_)]
    _oracle_exact(geo, case, kref, vref, "f32")
    for sumsq in (True, False):
        kp = [torch.zeros(nb, bs, n_kv, hd, device=cuda) for _ in range(L_)]
        vp = [torch.zeros(nb, bs, n_kv, hd, device=cuda) for _ in range(L_)]
        _run_exact(cuda, geo, case, rank, kp, vp, sumsq=sumsq)
        for l in range(L_):
            for got_t, ref in ((kp[l], kref[l]), (vp[l], vref[l])):
                err = rel_l2(got_t.cpu().numpy(), ref)
                assert err < REL_TOL, (sumsq, l, err)


LLAMA70B = dict(d=8192, n_kv=8, hd=128, theta=500000.0, lens=(4096, 1000, 17))


def _dense_case(seed, n_layers=2, bs=16):
    """The RL-step delta as the throughput run makes it: bf16 activations N(0, 1), full-rank
    dW_K, dW_V ~ N(0, (1e-3 * 0.02)^2) (||dW|| / ||W|| = 1e-3 for W ~ N(0, 0.02^2))."""
    geo = LLAMA70B
    g = torch.Generator().manual_seed(seed)
    d, d_kv = geo["d"], geo["n_kv"] * geo["hd"]
    lens = list(geo["lens"])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    rows = int(cu[-1])
    x = torch.randn(n_layers, rows, d, generator=g).to(torch.bfloat16)
    dw_k = (torch.randn(n_layers, d_kv, d, generator=g) * 2e-5).to(torch.bfloat16)
    dw_v = (torch.randn(n_layers, d_kv, d, generator=g) * 2e-5).to(torch.bfloat16)
    rng = np.random.default_rng(seed)
    tables, nb = _tables(rng, lens, bs)
    tabs = OX.rope_tables(geo["hd"], max(lens), geo["theta"])
    return dict(lens=lens, cu=cu, x=x, dw_k=dw_k, dw_v=dw_v, tables=tables, nb=nb, tabs=tabs, bs=bs, L=n_layers,
                rng=rng)


def _run_dense(cuda, case, k_pages, v_pages, accumulate=True):
    geo = LLAMA70B
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    patcher = dkv.DensePatcher(geo["d"], geo["n_kv"], geo["hd"],
                               rope=(torch.from_numpy(case["tabs"][0]), torch.from_numpy(case["tabs"][1])))
    packed = patcher.pack(case["dw_k"].to(cuda), case["dw_v"].to(cuda))
    seqs = ops.SeqBatchTensors(cu_seqlens=t(case["cu"]), block_tables=t(case["tables"]),
                               max_seq_len=max(case["lens"]))
    patcher.apply(case["x"].to(cuda), packed, k_pages, v_pages, seqs, accumulate=accumulate, check=True)
    torch.cuda.synchronize()


def _oracle_dense(case, k_pages, v_pages, kind, accumulate=True):
    geo = LLAMA70B
    OD.dense_patch_paged(x=case["x"].float().numpy(), norm_w=None, eps=1e-6, dw_k=case["dw_k"].float().numpy(),
                         dw_v=case["dw_v"].float().numpy(), cu_seqlens=case["cu"], block_tables=case["tables"],
                         k_pages=k_pages, v_pages=v_pages, n_kv=geo["n_kv"], hd=geo["hd"], rope=case["tabs"],
                         kind=kind, accumulate=accumulate)


def test_dense_bf16_pages_at_llama70b_geometry(cuda):
    case = _dense_case(31)
    geo = LLAMA70B
    L_, nb, bs, n_kv, hd = case["L"], case["nb"], case["bs"], geo["n_kv"], geo["hd"]
    # pages of the size of the delta (~2e-3) so that the delta moves most of them
    base = [[f32_to_bf16_bits(2e-3 * case["rng"].standard_normal((nb, bs, n_kv, hd), dtype=np.float32))
             for _ in range(L_)] for _kv in range(2)]
    kref = [b.copy() for b in base[0]]
    vref = [b.copy() for b in base[1]]
    _oracle_dense(case, kref, vref, "bf16")
    kp = [bf16_from_bits(b, cuda) for b in base[0]]
    vp = [bf16_from_bits(b, cuda) for b in base[1]]
    _run_dense(cuda, case, kp, vp)
    touched = _touched(nb, case["tables"], case["lens"], bs)
    for l in range(L_):
        for got_t, ref, inp in ((kp[l], kref[l], base[0][l]), (vp[l], vref[l], base[1][l])):
            got = bits_from_bf16(got_t)
            assert np.array_equal(got[~touched], inp[~touched])
            err = rel_l2(bf16_bits_to_f32(got[touched]), bf16_bits_to_f32(ref[touched]))
            assert err < REL_TOL, (l, err)
            eq = (got[touched] == ref[touched]).mean()
            assert eq >= BIT_EQUAL_MIN, (l, eq)


def test_dense_delta_f16_store_at_llama70b_geometry(cuda):
    """Store mode into f16 pages (11-bit significand, ~3e-4 rounding): the delta itself."""
    case = _dense_case(37)
    geo = LLAMA70B
    L_, nb, bs, n_kv, hd = case["L"], case["nb"], case["bs"], geo["n_kv"], geo["hd"]
    kref = [np.zeros((nb, bs, n_kv, hd), np.float32) for _ in range(L_)]
    vref = [np.zeros((nb, bs, n_kv, hd), np.float32) for _ in range(L_)]
    _oracle_dense(case, kref, vref, "f32", accumulate=False)
    kp = [torch.zeros(nb, bs, n_kv, hd, device=cuda, dtype=torch.float16) for _ in range(L_)]
    vp = [torch.zeros(nb, bs, n_kv, hd, device=cuda, dtype=torch.float16) for _ in range(L_)]
    _run_dense(cuda, case, kp, vp, accumulate=False)
    for l in range(L_):
        for got_t, ref in ((kp[l], kref[l]), (vp[l], vref[l])):
            err = rel_l2(got_t.float().cpu().numpy(), ref)
            assert err < REL_TOL, (l, err)
