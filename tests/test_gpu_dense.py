"""Dense-delta GEMM patch on the GPU vs the reference's golden vectors and the oracle.

The reference runs a dense dW through its exact route as LowRankFactors(A=dW, B=I);
the oracle restates that.  Tolerances: patched pages within rel-L2 1e-3 of the reference
result rounded to the page dtype (the required bar); in store mode (pages = delta) the
kernel's bf16 output within rel-L2 1e-3 of the oracle's delta rounded to bf16, with most
elements bit-identical (only fp32 summation order differs); untouched slots bit-identical.
Folding an RMSNorm weight into the packed bf16 dW rounds dW*w once to bf16, a relative
error of ~1e-3 of the delta (not of the pages).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deltakv_b200 as dkv
from deltakv_b200 import ops
from oracle import dense as OD
from oracle import exact as OX
from oracle.numerics import bf16_bits_to_f32
from tests.conftest import golden
from tests.helpers import bf16_from_bits, bits_from_bf16, rel_l2

pytestmark = pytest.mark.gpu
REL_TOL = 1e-3


def _touched_mask(nb: int, tables: np.ndarray, lens, bs: int) -> np.ndarray:
    m = np.zeros(nb, bool)
    for b, n in enumerate(lens):
        nblk = (int(n) + bs - 1) // bs
        m[tables[b, :nblk]] = True
    return m


def test_dense_paged_golden(cuda):
    """RMSNorm'd bf16 activations, full-rank dW_K / dW_V, RoPE, ragged batch, bf16 pages."""
    g = golden("dense_paged")
    n_kv, hd = int(g["n_kv"]), int(g["hd"])
    L_, rows, d = g["x_bits"].shape
    bs = int(g["block_size"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    patcher = dkv.DensePatcher(d, n_kv, hd, rope=(torch.from_numpy(g["rope_cos"]), torch.from_numpy(g["rope_sin"])),
                               norm_eps=float(g["eps"]))
    x = bf16_from_bits(g["x_bits"], cuda)
    packed = patcher.pack(bf16_from_bits(g["dw_k_bits"], cuda), bf16_from_bits(g["dw_v_bits"], cuda),
                          norm_weight=t(g["norm_w"]))
    xs = patcher.norm_scale(x)
    kp = [bf16_from_bits(g["k_pages_in"][l], cuda) for l in range(L_)]
    vp = [bf16_from_bits(g["v_pages_in"][l], cuda) for l in range(L_)]
    cu = g["cu_seqlens"]
    seqs = ops.SeqBatchTensors(cu_seqlens=t(cu), block_tables=t(g["block_tables"]), max_seq_len=int(np.diff(cu).max()))
    patcher.apply(x, packed, kp, vp, seqs, x_scale=xs, check=True)
    torch.cuda.synchronize()
    touched = _touched_mask(g["k_pages_in"].shape[1], g["block_tables"], np.diff(cu), bs)
    for l in range(L_):
        for got_t, ref_bits, in_bits in ((kp[l], g["k_pages_out"][l], g["k_pages_in"][l]),
                                         (vp[l], g["v_pages_out"][l], g["v_pages_in"][l])):
            got = bits_from_bf16(got_t)
            assert np.array_equal(got[~touched], in_bits[~touched])
            dg = bf16_bits_to_f32(got) - bf16_bits_to_f32(in_bits)
            dr = bf16_bits_to_f32(ref_bits) - bf16_bits_to_f32(in_bits)
            assert rel_l2(bf16_bits_to_f32(got), bf16_bits_to_f32(ref_bits)) < REL_TOL
            # the delta alone, with the bf16 rounding of both pages (~1e-2 of a delta of 20 % of the
            # page); the delta itself, stored into f16 pages, is held to 1e-3 of the oracle's fp32
            # x.dW^T at the Llama-70B shape (test_gpu_fullshape.py)
            assert rel_l2(dg, dr) < 2e-2
            assert (got == ref_bits).mean() > 0.95


def _tables(gen, lens, bs):
    need = [(n + bs - 1) // bs for n in lens]
    nb = sum(need) + 3
    perm = torch.randperm(nb, generator=gen).numpy().astype(np.int32)
    tables = np.zeros((len(lens), max(max(need), 1)), np.int32)
    k = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[k:k + n]
        k += n
    return tables, nb


@pytest.mark.parametrize(
    "d,n_kv,hd,bs,pdt,rope,do_k,do_v,acc,xscale,positions",
    [
        (256, 2, 128, 16, torch.bfloat16, True, True, True, False, False, False),
        (512, 8, 128, 16, torch.bfloat16, True, True, True, True, True, False),
        (576, 3, 64, 16, torch.bfloat16, True, True, True, False, False, False),   # 2*d_kv = 384: partial column block
        (192, 4, 32, 1, torch.float16, True, True, True, True, False, True),
        (128, 2, 64, 32, torch.bfloat16, False, True, True, False, True, False),
        (256, 4, 64, 16, torch.bfloat16, True, False, True, False, False, False),  # V only
        (256, 4, 64, 16, torch.float16, True, True, False, True, False, False),    # K only
        (64, 1, 128, 8, torch.bfloat16, True, True, True, True, False, True),
    ],
)
def test_dense_patch_matches_oracle(cuda, d, n_kv, hd, bs, pdt, rope, do_k, do_v, acc, xscale, positions):
    gen = torch.Generator().manual_seed(d * 17 + n_kv * 5 + hd + bs)
    L_ = 2
    lens = [1, 37, 128, 130, 0, 257]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    rows = int(cu[-1])
    d_kv = n_kv * hd
    x = (torch.randn(L_, rows, d, generator=gen) * 1.5).to(torch.bfloat16)
    dw_k = (torch.randn(L_, d_kv, d, generator=gen) * 0.03).to(torch.bfloat16)
    dw_v = (torch.randn(L_, d_kv, d, generator=gen) * 0.03).to(torch.bfloat16)
    xs = (torch.rand(L_, rows, generator=gen) + 0.5).float() if xscale else None
    tables, nb = _tables(gen, lens, bs)
    pos = None
    max_pos = max(lens) + 16
    if positions:
        pos = np.concatenate([np.arange(n) + 5 * b for b, n in enumerate(lens)]).astype(np.int32)
        max_pos = int(pos.max()) + 1
    tabs = OX.rope_tables(hd, max_pos, base=500000.0) if rope else None
    kind = {torch.bfloat16: "bf16", torch.float16: "f16"}[pdt]
    base_k = [torch.randn(nb, bs, n_kv, hd, generator=gen).to(pdt) for _ in range(L_)]
    base_v = [torch.randn(nb, bs, n_kv, hd, generator=gen).to(pdt) for _ in range(L_)]
    if not acc:
        base_k = [torch.zeros_like(p) for p in base_k]
        base_v = [torch.zeros_like(p) for p in base_v]
    to_np = (lambda tt: bits_from_bf16(tt)) if pdt == torch.bfloat16 else (lambda tt: tt.cpu().numpy())
    kref = [to_np(tt).copy() for tt in base_k]
    vref = [to_np(tt).copy() for tt in base_v]
    # oracle: the reference's exact route with A = dW, B = I, per (layer, sequence)
    xf = x.float().numpy()
    for l in range(L_):
        fk, fv = OD.dense_factors(dw_k[l].float().numpy() if do_k else None, dw_v[l].float().numpy() if do_v else None)
        for b in range(len(lens)):
            r0, r1 = int(cu[b]), int(cu[b + 1])
            if r1 == r0:
                continue
            xv = xf[l, r0:r1] * (xs[l, r0:r1].numpy()[:, None] if xs is not None else np.float32(1))
            p = None if pos is None else pos[r0:r1]
            dk, dv = OX.exact_kv_delta(xv.astype(np.float32), fk, fv, n_kv, hd, tabs, positions=p)
            tab = tables[b]
            for src, pg, on in ((dk, kref[l], do_k), (dv, vref[l], do_v)):
                if not on:
                    continue
                if acc:
                    OX.scatter_into_paged(src, pg, list(tab), bs, kind=kind)
                else:
                    for i in range(src.shape[0]):
                        pg[tab[i // bs], i % bs] = OX._from_f32(src[i], kind)
    # kernel
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    rope_t = (torch.from_numpy(tabs[0]), torch.from_numpy(tabs[1])) if rope else None
    patcher = dkv.DensePatcher(d, n_kv, hd, rope=rope_t)
    packed = patcher.pack(dw_k.to(cuda) if do_k else None, dw_v.to(cuda) if do_v else None)
    kp = [tt.to(cuda) for tt in base_k]
    vp = [tt.to(cuda) for tt in base_v]
    seqs = ops.SeqBatchTensors(cu_seqlens=t(cu), block_tables=t(tables), max_seq_len=max(lens),
                               positions=t(pos) if pos is not None else None)
    patcher.apply(x.to(cuda), packed, kp, vp, seqs, x_scale=xs.to(cuda) if xs is not None else None,
                  do_k=do_k, do_v=do_v, accumulate=acc, check=True)
    for l in range(L_):
        for got_t, ref in ((kp[l], kref[l]), (vp[l], vref[l])):
            got = to_np(got_t)
            if pdt == torch.bfloat16:
                a, b = bf16_bits_to_f32(got), bf16_bits_to_f32(ref)
            else:
                a, b = got.astype(np.float32), ref.astype(np.float32)
            if not np.any(b):
                assert not np.any(a)
                continue
            assert rel_l2(a, b) < REL_TOL, (l, rel_l2(a, b))
            assert (got == ref).mean() > 0.9


def test_row_inv_rms_matches_oracle(cuda):
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(300, 4096, generator=gen).to(torch.bfloat16)
    got = ops.row_inv_rms(x.to(cuda), 1e-5).cpu().numpy()
    xf = x.float().numpy()
    want = 1.0 / np.sqrt((xf.astype(np.float64) ** 2).mean(-1) + 1e-5)
    assert np.abs(got / want - 1).max() < 1e-5


def test_dense_errors_reported(cuda):
    patcher = dkv.DensePatcher(64, 1, 64, rope=(torch.ones(8, 32), torch.zeros(8, 32)))
    packed = patcher.pack(torch.randn(64, 64, device=cuda), torch.randn(64, 64, device=cuda))
    x = torch.randn(1, 20, 64, device=cuda).to(torch.bfloat16)
    kp = [torch.zeros(2, 16, 1, 64, device=cuda, dtype=torch.bfloat16)]
    vp = [torch.zeros(2, 16, 1, 64, device=cuda, dtype=torch.bfloat16)]
    seqs = ops.SeqBatchTensors(cu_seqlens=torch.tensor([0, 20], dtype=torch.int32, device=cuda),
                               block_tables=torch.tensor([[0, 1]], dtype=torch.int32, device=cuda), max_seq_len=20)
    with pytest.raises(dkv.DkvError, match="RoPE"):
        patcher.apply(x, packed, kp, vp, seqs, check=True)
    short = ops.SeqBatchTensors(cu_seqlens=torch.tensor([0, 20], dtype=torch.int32, device=cuda),
                                block_tables=torch.tensor([[0]], dtype=torch.int32, device=cuda), max_seq_len=20)
    nr = dkv.DensePatcher(64, 1, 64)
    with pytest.raises(dkv.DkvError, match="block_table"):
        nr.apply(x, packed, kp, vp, short, check=True)
    with pytest.raises(dkv.DkvError):
        dkv.DensePatcher(100, 1, 64).pack(torch.randn(64, 100, device=cuda), None)
