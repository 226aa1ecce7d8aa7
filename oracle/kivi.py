"""Oracle of the KIVI-style int4 KV format (numpy; TEST INFRASTRUCTURE ONLY).

The reference has no int4 cache; its only int4 arithmetic is the fake-quant
``metrics._minmax_quantize`` (src/deltakv/metrics.py:115-132): per group of 32 along the last
dimension, ``scale = max(hi - lo, 1e-8) / 15``, ``q = clamp(round((x - lo) / scale), 0, 15)``,
``deq = q * scale + lo``.  The stored format follows it with three choices of this build
(parity with the reference is therefore unpinned beyond ``tests/golden/kivi.npz``):

* V groups 32 consecutive channels of one token; K groups 32 consecutive tokens of one channel
  (a partial last group holds the remaining tokens);
* ``scale`` and ``lo`` are stored as fp16, rounded to nearest-even *before* q is computed
  (if the fp16 scale is 0, every q is 0);
* codes are packed two per byte along channels, the even channel in the low nibble:
  ``codes[t, c // 2]``; V scale/zero are ``[tokens, d/32]``, K scale/zero ``[ceil(n/32), d]``.

Every step is one IEEE fp32 operation (subtract, divide, multiply, add; ``rint`` ties to even)
so the CUDA kernels reproduce it bit for bit.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
G = 32


def _quant_groups(x: np.ndarray):
    """``x [..., 32]`` fp32 -> codes uint8 [..., 32], scale16, zero16 (float16 arrays)."""
    lo = x.min(axis=-1)
    hi = x.max(axis=-1)
    rng = np.maximum((hi - lo).astype(F32), F32(1e-8))
    scale16 = (rng / F32(15.0)).astype(F32).astype(np.float16)
    zero16 = lo.astype(np.float16)
    s = scale16.astype(F32)[..., None]
    z = zero16.astype(F32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint(((x - z).astype(F32) / s).astype(F32))
    q = np.where(s > 0, np.clip(q, 0, 15), 0).astype(np.uint8)
    return q, scale16, zero16


def _dequant(q: np.ndarray, scale16: np.ndarray, zero16: np.ndarray) -> np.ndarray:
    return ((q.astype(F32) * scale16.astype(F32)).astype(F32) + zero16.astype(F32)).astype(F32)


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """``q [n, d]`` (values 0..15) -> bytes ``[n, d/2]``, even channel in the low nibble."""
    return (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(b: np.ndarray) -> np.ndarray:
    n, h = b.shape
    q = np.empty((n, 2 * h), np.uint8)
    q[:, 0::2] = b & 0xF
    q[:, 1::2] = b >> 4
    return q


def quantize(x: np.ndarray, mode: str):
    """``x [n, d]`` -> ``(codes [n, d/2] uint8, scale, zero)``; mode "v" (per token) or "k"."""
    x = np.asarray(x, F32)
    n, d = x.shape
    if d % G:
        raise ValueError("d must be a multiple of 32")
    if mode == "v":
        q, s, z = _quant_groups(x.reshape(n, d // G, G))
        return pack_nibbles(q.reshape(n, d)), s, z
    ng = (n + G - 1) // G
    q = np.zeros((n, d), np.uint8)
    s = np.zeros((ng, d), np.float16)
    z = np.zeros((ng, d), np.float16)
    for gi in range(ng):
        t0, t1 = gi * G, min(n, gi * G + G)
        qq, ss, zz = _quant_groups(x[t0:t1].T)  # [d, tokens]
        q[t0:t1] = qq.T
        s[gi], z[gi] = ss, zz
    return pack_nibbles(q), s, z


def dequantize(codes: np.ndarray, scale: np.ndarray, zero: np.ndarray, mode: str) -> np.ndarray:
    q = unpack_nibbles(codes)
    n, d = q.shape
    if mode == "v":
        return _dequant(q.reshape(n, d // G, G), scale[..., None], zero[..., None]).reshape(n, d)
    rows = np.arange(n) // G
    return _dequant(q, scale[rows], zero[rows])


def patch(codes, scale, zero, delta: np.ndarray, mode: str):
    """dequant -> + delta (fp32) -> requant: the KIVI form of a KV patch."""
    x = (dequantize(codes, scale, zero, mode) + np.asarray(delta, F32)).astype(F32)
    return quantize(x, mode)
