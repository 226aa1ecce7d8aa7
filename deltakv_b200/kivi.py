"""KIVI-style int4 KV caches on the B200 kernels.

K tensors use per-channel groups (32 consecutive tokens of a channel), V tensors per-token
groups (32 consecutive channels); asymmetric min-max with fp16 scale and zero, two codes per
byte.  The reference keeps caches in the model dtype and only fake-quantises them to report
a noise floor (metrics._minmax_quantize, src/deltakv/metrics.py:115-132); this is the stored
counterpart, so a patch can be applied as dequant -> add -> requant in one pass.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
from torch import Tensor

from deltakv_b200 import _lib as L
from deltakv_b200 import ops

GROUP = 32


@dataclass
class KiviTensor:
    """One int4 K or V tensor of ``n_tokens x d``."""

    codes: Tensor  # uint8 [n, d/2]
    scale: Tensor  # fp16, V: [n, d/32], K: [ceil(n/32), d]
    zero: Tensor
    mode: str      # "k" (per channel) or "v" (per token)

    @property
    def n_tokens(self) -> int:
        return int(self.codes.shape[0])

    @property
    def d(self) -> int:
        return int(self.codes.shape[1]) * 2

    @staticmethod
    def empty(n_tokens: int, d: int, mode: str, device) -> "KiviTensor":
        if d % GROUP:
            raise ValueError("d must be a multiple of 32")
        codes = torch.empty(n_tokens, d // 2, dtype=torch.uint8, device=device)
        if mode == "v":
            shape = (n_tokens, d // GROUP)
        elif mode == "k":
            shape = ((n_tokens + GROUP - 1) // GROUP, d)
        else:
            raise ValueError("mode must be 'k' or 'v'")
        return KiviTensor(codes, torch.empty(shape, dtype=torch.float16, device=device),
                          torch.empty(shape, dtype=torch.float16, device=device), mode)

    def desc(self) -> L.KiviCache:
        ops._require_cuda(self.codes, self.scale, self.zero)
        if self.scale.stride() != self.zero.stride() or self.scale.stride(1) != 1 or self.codes.stride(1) != 1:
            raise ValueError("scale/zero must share a row-major layout; codes rows contiguous")
        return L.KiviCache(
            codes=self.codes.data_ptr(), scale=self.scale.data_ptr(), zero=self.zero.data_ptr(),
            code_row_stride=self.codes.stride(0), sz_row_stride=self.scale.stride(0),
            n_tokens=self.n_tokens, d=self.d,
            mode=L.DKV_KIVI_PER_CHANNEL if self.mode == "k" else L.DKV_KIVI_PER_TOKEN,
        )


def _rows(x: Tensor) -> Tensor:
    x2 = x.reshape(x.shape[0], -1)
    return x2 if x2.stride(1) == 1 else x2.contiguous()


def quantize(x: Tensor, mode: str) -> KiviTensor:
    """``x [n, ...]`` (fp32/bf16/f16) -> int4 with the K ("k") or V ("v") grouping."""
    x2 = _rows(x)
    out = KiviTensor.empty(x2.shape[0], x2.shape[1], mode, x2.device)
    desc = out.desc()
    rc = L.lib().dkv_kivi_quantize(x2.data_ptr(), ops.dkv_dtype(x2.dtype), x2.stride(0), C.byref(desc),
                                   ops.stream_ptr())
    L.check(rc, "dkv_kivi_quantize")
    return out


def dequantize(t: KiviTensor, dtype: torch.dtype = torch.float32) -> Tensor:
    out = torch.empty(t.n_tokens, t.d, dtype=dtype, device=t.codes.device)
    desc = t.desc()
    rc = L.lib().dkv_kivi_dequantize(C.byref(desc), out.data_ptr(), ops.dkv_dtype(dtype), out.stride(0),
                                     ops.stream_ptr())
    L.check(rc, "dkv_kivi_dequantize")
    return out


def patch(base: KiviTensor, delta: Tensor | None, out: KiviTensor | None = None) -> KiviTensor:
    """``out = int4(dequant(base) + delta)``; ``out=None`` patches ``base`` in place."""
    out = base if out is None else out
    bd, od = base.desc(), out.desc()
    dptr, ddt, drs = None, 0, 0
    if delta is not None:
        d2 = _rows(delta)
        ops._require_cuda(d2)
        dptr, ddt, drs = d2.data_ptr(), ops.dkv_dtype(d2.dtype), d2.stride(0)
    rc = L.lib().dkv_kivi_patch(C.byref(bd), dptr, ddt, drs, C.byref(od), ops.stream_ptr())
    L.check(rc, "dkv_kivi_patch")
    return out
