"""Tensor-level wrappers over the C ABI.

These functions take CUDA tensors, describe them to the library (base pointer, dtype,
element strides), launch on the current torch stream and return.  Nothing here computes
on the CPU; a non-CUDA tensor is an error.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Sequence

import torch

from deltakv_b200 import _lib as L

_DT = {torch.float32: L.DKV_F32, torch.float16: L.DKV_F16, torch.bfloat16: L.DKV_BF16}
if hasattr(torch, "float8_e4m3fn"):
    _DT[torch.float8_e4m3fn] = L.DKV_E4M3


def dkv_dtype(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise TypeError(f"dtype {t} is not supported by the B200 kernels") from None


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("deltakv_b200 kernels need CUDA tensors (there is no CPU path)")


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# paged cache descriptors
# ---------------------------------------------------------------------------
def page_view(cache: torch.Tensor, kv_dim: int = 0) -> torch.Tensor:
    """Select the ``[num_blocks, block_size, n_heads, head_dim]`` view the reference writes.

    Mirrors the layout dispatch of ``scatter_into_paged`` (src/deltakv/paged.py:18-37),
    including its error text.
    """
    if cache.ndim == 4:
        return cache
    if cache.ndim == 5 and cache.shape[0] == 2:
        return cache[kv_dim]
    if cache.ndim == 5 and cache.shape[1] == 2:
        return cache[:, kv_dim]
    raise ValueError(f"unsupported paged KV layout {tuple(cache.shape)}")


def paged_desc(pages: torch.Tensor) -> L.PagedCache:
    """Describe a ``[num_blocks, block_size, n_heads, head_dim]`` (possibly strided) view."""
    _require_cuda(pages)
    if pages.ndim != 4:
        raise ValueError(f"unsupported paged KV layout {tuple(pages.shape)}")
    if pages.stride(3) != 1:
        raise ValueError("paged cache head_dim must be contiguous")
    nb, bs, h, d = pages.shape
    return L.PagedCache(
        base=pages.data_ptr(),
        dtype=dkv_dtype(pages.dtype),
        block_size=bs,
        n_heads=h,
        head_dim=d,
        num_blocks=nb,
        stride_block=pages.stride(0),
        stride_slot=pages.stride(1),
        stride_head=pages.stride(2),
    )


@dataclass
class SeqBatchTensors:
    """Device-side description of a batch of sequences (kept alive with the struct)."""

    cu_seqlens: torch.Tensor  # int32 [n_seqs+1]
    block_tables: torch.Tensor  # int32 [n_seqs, max_blocks]
    max_seq_len: int
    table_lens: torch.Tensor | None = None
    positions: torch.Tensor | None = None

    def __post_init__(self):
        bt = self.block_tables
        if self.table_lens is None and bt.ndim == 2 and bt.shape[0] > 0 and bt.stride(0) != bt.shape[1]:
            # Without per-row lengths the C ABI takes a row's length from the row stride, so
            # the rows get standard strides here (numpy's x[None] gives a one-row table row
            # stride 0; a column slice has a stride above its width).  Kept in the dataclass,
            # the copy lives as long as the launches that read it.
            self.block_tables = torch.empty(bt.shape, dtype=bt.dtype, device=bt.device).copy_(bt)

    def struct(self) -> L.SeqBatch:
        _require_cuda(self.cu_seqlens, self.block_tables, self.table_lens, self.positions)
        for t in (self.cu_seqlens, self.block_tables, self.table_lens, self.positions):
            if t is not None and t.dtype != torch.int32:
                raise TypeError("sequence metadata must be int32")
        bt = self.block_tables
        if bt.ndim != 2 or bt.stride(1) != 1:
            raise ValueError("block_tables must be a row-major [n_seqs, max_blocks] int32 tensor")
        return L.SeqBatch(
            cu_seqlens=self.cu_seqlens.data_ptr(),
            block_tables=bt.data_ptr(),
            table_lens=ptr(self.table_lens),
            positions=ptr(self.positions),
            table_stride=bt.stride(0),
            n_seqs=self.cu_seqlens.numel() - 1,
            max_seq_len=int(self.max_seq_len),
        )

    @staticmethod
    def single(seq_len: int, block_table: Sequence[int], device: torch.device) -> "SeqBatchTensors":
        """One sequence with a Python block table (the reference's calling convention)."""
        cu = torch.tensor([0, seq_len], dtype=torch.int32, device=device)
        bt = torch.tensor([list(block_table)] if len(block_table) else [[0]], dtype=torch.int32)
        return SeqBatchTensors(
            cu_seqlens=cu,
            block_tables=bt.to(device),
            max_seq_len=seq_len,
            table_lens=torch.tensor([len(block_table)], dtype=torch.int32, device=device),
        )


class StatusWord:
    """A device int32 that kernels set to the first error they meet."""

    def __init__(self, device: torch.device):
        self.t = torch.zeros(1, dtype=torch.int32, device=device)

    @property
    def ptr(self) -> int:
        return self.t.data_ptr()

    def raise_if_set(self, where: str) -> None:
        code = int(self.t.item())
        if code != 0:
            self.t.zero_()
            raise L.DkvError(code, where)


_status_words: dict[int, StatusWord] = {}


def status_word(device: torch.device) -> StatusWord:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _status_words:
        _status_words[idx] = StatusWord(torch.device("cuda", idx))
    return _status_words[idx]


# ---------------------------------------------------------------------------
# scatter / gather
# ---------------------------------------------------------------------------
def scatter_paged(delta: torch.Tensor, pages: torch.Tensor, seqs: SeqBatchTensors,
                  status: StatusWord | None = None) -> None:
    """``pages[block(t), slot(t)] += delta[t]`` for the rows of every sequence."""
    _require_cuda(delta, pages)
    if delta.ndim != 3 or delta.stride(2) != 1:
        raise ValueError("delta must be [rows, n_heads, head_dim] with contiguous head_dim")
    desc = paged_desc(pages)
    sb = seqs.struct()
    rc = L.lib().dkv_scatter_paged(
        delta.data_ptr(), dkv_dtype(delta.dtype), delta.stride(0), delta.stride(1),
        C.byref(desc), C.byref(sb), status.ptr if status else None, stream_ptr(),
    )
    L.check(rc, "dkv_scatter_paged")


def gather_paged(pages: torch.Tensor, seqs: SeqBatchTensors, out: torch.Tensor,
                 status: StatusWord | None = None) -> torch.Tensor:
    _require_cuda(pages, out)
    desc = paged_desc(pages)
    sb = seqs.struct()
    rc = L.lib().dkv_gather_paged(
        C.byref(desc), C.byref(sb), out.data_ptr(), dkv_dtype(out.dtype), out.stride(0),
        out.stride(1), status.ptr if status else None, stream_ptr(),
    )
    L.check(rc, "dkv_gather_paged")
    return out


# ---------------------------------------------------------------------------
# stored-activation format
# ---------------------------------------------------------------------------
def quantize_rows(x: torch.Tensor, out_dtype: torch.dtype = torch.float16,
                  pad_to: int = 16, with_sumsq: bool = False):
    """``x [..., rows, d]`` (fp32/bf16/f16) -> ``(q [..., rows, d_pad], scale [..., rows])``
    with ``x ~= q * scale``; ``d_pad`` rounds ``d`` up so a row is a multiple of 16 bytes
    (the padding is zero).  ``with_sumsq`` adds ``sumsq [..., rows]``, each row's sum of
    squared stored codes, for the exact patch's RMSNorm (``ExactPatcher.apply(x_sumsq=...)``)."""
    _require_cuda(x)
    lead = x.shape[:-1]
    d = x.shape[-1]
    x2 = x.reshape(-1, d)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    esz = 1 if out_dtype != torch.float16 else 2
    step = max(1, pad_to // esz)
    d_pad = (d + step - 1) // step * step
    q = torch.empty(x2.shape[0], d_pad, dtype=out_dtype, device=x.device)
    scale = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
    sumsq = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device) if with_sumsq else None
    rc = L.lib().dkv_quantize_rows_sumsq(
        x2.data_ptr(), dkv_dtype(x2.dtype), x2.shape[0], d, x2.stride(0), q.data_ptr(),
        dkv_dtype(out_dtype), q.stride(0), d_pad, scale.data_ptr(), ptr(sumsq), stream_ptr(),
    )
    L.check(rc, "dkv_quantize_rows_sumsq")
    if with_sumsq:
        return q.view(*lead, d_pad), scale.view(*lead), sumsq.view(*lead)
    return q.view(*lead, d_pad), scale.view(*lead)


# ---------------------------------------------------------------------------
# exact patch
# ---------------------------------------------------------------------------
def exact_geometry(d_model: int, n_kv_heads: int, head_dim: int, x_dtype: torch.dtype,
                   rank_k: int, rank_v: int) -> L.ExactGeometry:
    return L.ExactGeometry(d_model=d_model, n_kv_heads=n_kv_heads, head_dim=head_dim,
                           x_dtype=dkv_dtype(x_dtype), rank_k=rank_k, rank_v=rank_v)


def packed_bytes(geom: L.ExactGeometry) -> int:
    out = C.c_int64(0)
    L.check(L.lib().dkv_exact_packed_bytes(C.byref(geom), C.byref(out)), "dkv_exact_packed_bytes")
    return int(out.value)


def pack_factors(geom: L.ExactGeometry, a_k: torch.Tensor | None, b_k: torch.Tensor | None,
                 a_v: torch.Tensor | None, b_v: torch.Tensor | None, scale_k: float,
                 scale_v: float, norm_weight: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Pack per-layer LoRA factors ``A [L, r, d]``, ``B [L, d_kv, r]`` (or unbatched)
    into the kernel's operand image; returns a uint8 tensor ``[L, bytes_per_layer]``."""
    mats = [m for m in (a_k, b_k, a_v, b_v) if m is not None]
    if not mats:
        raise ValueError("no factors to pack")
    dev = mats[0].device
    _require_cuda(*mats, norm_weight)
    dt = mats[0].dtype
    def prep(m):
        if m is None:
            return None
        m = m if m.ndim == 3 else m.unsqueeze(0)
        return m.to(dt).contiguous()
    a_k, b_k, a_v, b_v = prep(a_k), prep(b_k), prep(a_v), prep(b_v)
    n_layers = (a_k if a_k is not None else a_v).shape[0]
    nbytes = packed_bytes(geom)
    if out is None:
        out = torch.empty(n_layers, nbytes, dtype=torch.uint8, device=dev)
    nw = None
    if norm_weight is not None:
        nw = (norm_weight if norm_weight.ndim == 2 else norm_weight.unsqueeze(0)).contiguous()
    f = L.LoraFactors(
        a_k=ptr(a_k), b_k=ptr(b_k), a_v=ptr(a_v), b_v=ptr(b_v), dtype=dkv_dtype(dt),
        rank_k=geom.rank_k, rank_v=geom.rank_v, n_layers=n_layers,
        scale_k=float(scale_k), scale_v=float(scale_v),
        a_k_layer_stride=a_k.stride(0) if a_k is not None else 0,
        b_k_layer_stride=b_k.stride(0) if b_k is not None else 0,
        a_v_layer_stride=a_v.stride(0) if a_v is not None else 0,
        b_v_layer_stride=b_v.stride(0) if b_v is not None else 0,
        norm_weight=ptr(nw), norm_dtype=dkv_dtype(nw.dtype) if nw is not None else 0,
        norm_layer_stride=nw.stride(0) if (nw is not None and nw.shape[0] > 1) else 0,
    )
    rc = L.lib().dkv_pack_exact_factors(C.byref(geom), C.byref(f), out.data_ptr(),
                                        out.stride(0), stream_ptr())
    L.check(rc, "dkv_pack_exact_factors")
    return out


def exact_patch_paged(geom: L.ExactGeometry, x: torch.Tensor, packed: torch.Tensor,
                      k_pages: Sequence[torch.Tensor], v_pages: Sequence[torch.Tensor],
                      seqs: SeqBatchTensors, *, x_scale: torch.Tensor | None = None,
                      apply_norm: bool = False, norm_eps: float = 1e-6,
                      rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
                      accumulate: bool = True, status: StatusWord | None = None,
                      x_sumsq: torch.Tensor | None = None) -> None:
    """Launch the fused patch over ``L = len(k_pages)`` layers.

    ``x`` is ``[L, rows, d]`` (or ``[rows, d]`` for one layer) in fp8-e4m3 or f16;
    ``x_scale`` ``[L, rows]`` fp32; ``k_pages[l]`` / ``v_pages[l]`` are
    ``[num_blocks, block_size, n_kv, head_dim]`` views; ``rope_cos/sin`` are
    ``[max_pos, head_dim/2]`` fp32 tables.  ``x_sumsq`` ``[L, rows]`` fp32 (from
    :func:`quantize_rows` ``with_sumsq``): with ``apply_norm`` the RMSNorm takes each row's
    sum of squared codes from it instead of forming it on the tensor cores.
    """
    n_layers = len(k_pages)
    if len(v_pages) != n_layers:
        raise ValueError("k_pages and v_pages must cover the same layers")
    if n_layers > L.DKV_MAX_LAYERS:
        raise ValueError(f"at most {L.DKV_MAX_LAYERS} layers per launch")
    x3 = x if x.ndim == 3 else x.unsqueeze(0)
    if x3.shape[0] != n_layers:
        raise ValueError("x layers do not match the page lists")
    _require_cuda(x3, packed, x_scale, rope_cos, rope_sin, x_sumsq)
    if x3.stride(2) != 1:
        raise ValueError("x rows must be contiguous")
    xs = None
    if x_scale is not None:
        xs = x_scale if x_scale.ndim == 2 else x_scale.unsqueeze(0)
        if xs.dtype != torch.float32 or xs.stride(1) != 1:
            raise TypeError("x_scale must be fp32 with contiguous rows")
    xq = None
    if x_sumsq is not None:
        if not apply_norm:
            raise ValueError("x_sumsq feeds the RMSNorm: pass it only with apply_norm=True")
        xq = x_sumsq if x_sumsq.ndim == 2 else x_sumsq.unsqueeze(0)
        if xq.dtype != torch.float32:
            raise TypeError("x_sumsq must be fp32")
        if xq.stride(1) != 1 or xq.shape[0] != n_layers or xq.shape[1] < x3.shape[1]:
            raise ValueError("x_sumsq must be [layers, rows] with contiguous rows, matching x")
    kd = (L.PagedCache * n_layers)(*[paged_desc(p) for p in k_pages])
    vd = (L.PagedCache * n_layers)(*[paged_desc(p) for p in v_pages])
    if rope_cos is not None:
        rope_cos = rope_cos.contiguous()
        rope_sin = rope_sin.contiguous()
    args = L.ExactPatchArgs(
        geom=geom,
        x=x3.data_ptr(), x_layer_stride=x3.stride(0), x_row_stride=x3.stride(1),
        x_rows=x3.shape[1],
        x_scale=ptr(xs), x_scale_layer_stride=xs.stride(0) if xs is not None else 0,
        apply_norm=1 if apply_norm else 0, norm_eps=float(norm_eps),
        packed=packed.data_ptr(), packed_layer_stride=packed.stride(0) if packed.ndim == 2 else 0,
        rope_cos=ptr(rope_cos), rope_sin=ptr(rope_sin),
        rope_max_pos=rope_cos.shape[0] if rope_cos is not None else 0,
        n_layers=n_layers,
        seqs=seqs.struct(),
        k_pages=kd, v_pages=vd,
        accumulate=1 if accumulate else 0,
        status=status.ptr if status else None,
        x_sumsq=ptr(xq), x_sumsq_layer_stride=xq.stride(0) if xq is not None else 0,
    )
    rc = L.lib().dkv_exact_patch_paged(C.byref(args), stream_ptr())
    L.check(rc, "dkv_exact_patch_paged")


# ---------------------------------------------------------------------------------------
# dense-delta route
# ---------------------------------------------------------------------------------------
def dense_geometry(d_model: int, n_kv_heads: int, head_dim: int) -> L.DenseGeometry:
    return L.DenseGeometry(d_model=d_model, n_kv_heads=n_kv_heads, head_dim=head_dim)


def pack_dense_delta(geom: L.DenseGeometry, dw_k: torch.Tensor | None, dw_v: torch.Tensor | None,
                     *, scale_k: float = 1.0, scale_v: float = 1.0,
                     norm_weight: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``dw_k``/``dw_v``: ``[L, n_kv*hd, d]`` (or 2-D for one layer) -> bf16 ``[L, 2*n_kv*hd, d]``."""
    ref = dw_k if dw_k is not None else dw_v
    if ref is None:
        raise ValueError("at least one of dw_k / dw_v is required")
    d_kv = geom.n_kv_heads * geom.head_dim

    def as3(t):
        if t is None:
            return None
        t = t if t.ndim == 3 else t.unsqueeze(0)
        if tuple(t.shape[1:]) != (d_kv, geom.d_model):
            raise ValueError(f"dW shape {tuple(t.shape[1:])} != ({d_kv}, {geom.d_model})")
        return t.contiguous()

    k3, v3 = as3(dw_k), as3(dw_v)
    if k3 is not None and v3 is not None and (k3.dtype != v3.dtype or k3.shape[0] != v3.shape[0]):
        raise ValueError("dw_k and dw_v must share dtype and layer count")
    r3 = k3 if k3 is not None else v3
    n_layers = r3.shape[0]
    _require_cuda(k3, v3, norm_weight)
    nw = None
    if norm_weight is not None:
        nw = (norm_weight if norm_weight.ndim == 2 else norm_weight.unsqueeze(0).expand(n_layers, -1)).contiguous()
    if out is None:
        out = torch.empty(n_layers, 2 * d_kv, geom.d_model, dtype=torch.bfloat16, device=r3.device)
    dw = L.DenseDelta(
        dw_k=ptr(k3), dw_v=ptr(v3), dtype=dkv_dtype(r3.dtype), n_layers=n_layers,
        dw_k_layer_stride=k3.stride(0) if k3 is not None else 0,
        dw_v_layer_stride=v3.stride(0) if v3 is not None else 0,
        norm_weight=ptr(nw), norm_dtype=dkv_dtype(nw.dtype) if nw is not None else 0,
        norm_layer_stride=nw.stride(0) if nw is not None else 0,
        scale_k=float(scale_k), scale_v=float(scale_v),
    )
    rc = L.lib().dkv_pack_dense_delta(C.byref(geom), C.byref(dw), out.data_ptr(), out.stride(0), stream_ptr())
    L.check(rc, "dkv_pack_dense_delta")
    return out


def row_inv_rms(x: torch.Tensor, eps: float) -> torch.Tensor:
    """``1/sqrt(mean(x^2) + eps)`` per row of ``x [..., d]`` (fp32), the RMSNorm row factor."""
    _require_cuda(x)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
    rc = L.lib().dkv_row_inv_rms(x2.data_ptr(), dkv_dtype(x2.dtype), x2.shape[0], x2.shape[1], x2.stride(0),
                                 float(eps), out.data_ptr(), stream_ptr())
    L.check(rc, "dkv_row_inv_rms")
    return out.view(x.shape[:-1])


def dense_patch_paged(geom: L.DenseGeometry, x: torch.Tensor, packed: torch.Tensor,
                      k_pages: Sequence[torch.Tensor], v_pages: Sequence[torch.Tensor],
                      seqs: SeqBatchTensors, *, x_scale: torch.Tensor | None = None,
                      rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
                      do_k: bool = True, do_v: bool = True, accumulate: bool = True,
                      status: StatusWord | None = None) -> None:
    """Launch the dense-delta GEMM patch over ``L = len(k_pages)`` layers.

    ``x`` ``[L, rows, d]`` bf16; ``packed`` from :func:`pack_dense_delta`; ``x_scale``
    ``[L, rows]`` fp32 multiplies each row's product (e.g. the RMSNorm factor).
    """
    n_layers = len(k_pages)
    if len(v_pages) != n_layers:
        raise ValueError("k_pages and v_pages must cover the same layers")
    if n_layers > L.DKV_MAX_LAYERS:
        raise ValueError(f"at most {L.DKV_MAX_LAYERS} layers per launch")
    x3 = x if x.ndim == 3 else x.unsqueeze(0)
    if x3.shape[0] != n_layers:
        raise ValueError("x layers do not match the page lists")
    if x3.dtype != torch.bfloat16:
        raise TypeError("the dense route reads bf16 activations")
    p3 = packed if packed.ndim == 3 else packed.unsqueeze(0)
    if p3.shape[0] < n_layers or p3.dtype != torch.bfloat16:
        raise ValueError("packed delta must be bf16 [L, 2*n_kv*hd, d] covering every layer")
    _require_cuda(x3, p3, x_scale, rope_cos, rope_sin)
    if x3.stride(2) != 1 or p3.stride(2) != 1:
        raise ValueError("x and packed rows must be contiguous")
    xs = None
    if x_scale is not None:
        xs = x_scale if x_scale.ndim == 2 else x_scale.unsqueeze(0)
        if xs.dtype != torch.float32 or xs.stride(1) != 1:
            raise TypeError("x_scale must be fp32 with contiguous rows")
    kd = (L.PagedCache * n_layers)(*[paged_desc(p) for p in k_pages])
    vd = (L.PagedCache * n_layers)(*[paged_desc(p) for p in v_pages])
    if rope_cos is not None:
        rope_cos = rope_cos.contiguous()
        rope_sin = rope_sin.contiguous()
    args = L.DensePatchArgs(
        geom=geom,
        x=x3.data_ptr(), x_layer_stride=x3.stride(0), x_row_stride=x3.stride(1), x_rows=x3.shape[1],
        x_scale=ptr(xs), x_scale_layer_stride=xs.stride(0) if xs is not None else 0,
        packed=p3.data_ptr(), packed_layer_stride=p3.stride(0),
        rope_cos=ptr(rope_cos), rope_sin=ptr(rope_sin),
        rope_max_pos=rope_cos.shape[0] if rope_cos is not None else 0,
        n_layers=n_layers, do_k=1 if do_k else 0, do_v=1 if do_v else 0,
        seqs=seqs.struct(), k_pages=kd, v_pages=vd,
        accumulate=1 if accumulate else 0,
        status=status.ptr if status else None,
    )
    rc = L.lib().dkv_dense_patch_paged(C.byref(args), stream_ptr())
    L.check(rc, "dkv_dense_patch_paged")
