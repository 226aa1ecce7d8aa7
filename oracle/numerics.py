"""Bit-level number formats for the oracle (numpy; TEST INFRASTRUCTURE ONLY).

* bf16: the upper 16 bits of an IEEE fp32, rounded to nearest-even — what
  ``tensor.to(torch.bfloat16)`` does and what the reference's bf16 page store does
  (src/deltakv/paged.py:43 assigns an fp32 sum into a bf16 page).
* float8 e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; no infinities; S.1111.111
  is NaN; largest finite 448 (OCP FP8 specification).  The reference has no fp8; this is
  the stored-activation format of the B200 path.
"""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    r = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _e4m3_table() -> np.ndarray:
    tab = np.zeros(256, dtype=np.float32)
    for v in range(256):
        s = -1.0 if v & 0x80 else 1.0
        e = (v >> 3) & 0xF
        m = v & 0x7
        if e == 0xF and m == 0x7:
            tab[v] = np.nan
        elif e == 0:
            tab[v] = s * (m / 8.0) * 2.0 ** (-6)
        else:
            tab[v] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return tab


E4M3_TABLE = _e4m3_table()


def e4m3_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(b, dtype=np.uint8)]


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """Round to the nearest e4m3 value (ties to even), saturating at ±448."""
    x = np.asarray(x, dtype=np.float32)
    finite = E4M3_TABLE.copy()
    finite[np.isnan(finite)] = np.inf
    pos_codes = np.arange(0, 127, dtype=np.uint8)  # 0x00..0x7E, ascending values
    pos_vals = finite[pos_codes]
    a = np.minimum(np.abs(x), 448.0)
    idx = np.searchsorted(pos_vals, a)  # first value >= a
    idx = np.clip(idx, 1, len(pos_vals) - 1)
    lo, hi = pos_vals[idx - 1], pos_vals[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & ((pos_codes[idx] & 1) == 0))
    code = np.where(pick_hi, pos_codes[idx], pos_codes[idx - 1]).astype(np.uint8)
    code = np.where(a == 0, np.uint8(0), code)
    return np.where(np.signbit(x), code | np.uint8(0x80), code).astype(np.uint8)
