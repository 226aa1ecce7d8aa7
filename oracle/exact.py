"""Oracle of the exact / zeroth-order patch route and of the paged scatter/gather
(numpy fp32; TEST INFRASTRUCTURE ONLY).

Each function restates the reference's torch code, operation by operation:

* ``rope_tables``         RotaryEmbedding.__init__      src/deltakv/rope.py:28-45
* ``apply_rope``          apply_rope / rotate_half      src/deltakv/rope.py:9-25,55-63
* ``rmsnorm``             RMSNorm.forward               src/deltakv/model.py:48-56
* ``lora_codes/apply``    LowRankFactors.codes/.apply   src/deltakv/deltas/factors.py:61-67
* ``exact_kv_delta``      exact_kv_patch + materialize  src/deltakv/patches/exact.py:14-63,
                                                        src/deltakv/patches/tensors.py:105-123
* ``scatter_into_paged``  scatter_into_paged            src/deltakv/paged.py:8-43
* ``gather_from_paged``   gather_from_paged             src/deltakv/paged.py:46-70
* ``exact_patch_paged``   the engine's exact branch over many (layer, sequence) pairs
                          (engine.py:263-288 -> rmsnorm_tensors -> zeroth_order_patches ->
                          apply_layer_patches -> DeltaKVConnector.patch_paged's scatter)
"""

from __future__ import annotations

import numpy as np

from oracle.numerics import bf16_bits_to_f32, e4m3_bits_to_f32, f32_to_bf16_bits

F32 = np.float32


def rope_tables(head_dim: int, max_seq: int, base: float = 10000.0) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin of ``position * inv_freq`` for the first half of head_dim, ``[max_seq, hd/2]``.

    rope.py:35-45 builds ``emb = cat(freqs, freqs)``; both halves are equal, so the first
    half carries all the information.
    """
    if head_dim % 2:
        raise ValueError("RoPE head_dim must be even")
    inv_freq = (F32(1.0) / (F32(base) ** (np.arange(0, head_dim, 2, dtype=F32) / F32(head_dim)))).astype(F32)
    t = np.arange(max_seq, dtype=F32)
    freqs = np.outer(t, inv_freq).astype(F32)
    # cos/sin evaluated in float64 and rounded once to fp32
    return np.cos(freqs.astype(np.float64)).astype(F32), np.sin(freqs.astype(np.float64)).astype(F32)


def apply_rope(x: np.ndarray, cos_half: np.ndarray, sin_half: np.ndarray, positions: np.ndarray) -> np.ndarray:
    """``x [seq, heads, hd]`` rotated at ``positions`` (rotate-half pairing i <-> i+hd/2)."""
    hd = x.shape[-1]
    c = np.concatenate([cos_half, cos_half], axis=-1)[positions][:, None, :]
    s = np.concatenate([sin_half, sin_half], axis=-1)[positions][:, None, :]
    x1, x2 = x[..., : hd // 2], x[..., hd // 2 :]
    rot = np.concatenate([-x2, x1], axis=-1)
    return (x * c + rot * s).astype(F32)


def rmsnorm(x: np.ndarray, w: np.ndarray | None, eps: float) -> np.ndarray:
    """``x * rsqrt(mean(x^2) + eps) * w`` in fp32, multiplied in that order (model.py:55-56)."""
    y = np.array(x, dtype=F32, copy=True)
    ms = np.einsum("ij,ij->i", y, y, dtype=F32) / F32(y.shape[-1])
    r = (F32(1.0) / np.sqrt(ms + F32(eps))).astype(F32)
    y *= r[:, None]
    if w is not None:
        y *= w.astype(F32)
    return y


def lora_codes(x: np.ndarray, A: np.ndarray, scale: float) -> np.ndarray:
    return (F32(scale) * (x.astype(F32) @ A.astype(F32).T)).astype(F32)


def lora_apply(x: np.ndarray, A: np.ndarray, B: np.ndarray, scale: float) -> np.ndarray:
    return (lora_codes(x, A, scale) @ B.astype(F32).T).astype(F32)


def exact_kv_delta(x_normed: np.ndarray, fk, fv, n_kv: int, hd: int, rope=None,
                   positions: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """``(dK, dV)`` as ``[seq, n_kv, hd]`` fp32.  ``fk``/``fv`` are ``(A, B, scale)`` or
    None (missing projection -> zeros, exact.py:46-53).  ``rope`` is ``(cos, sin)`` halves
    or None (no positional keys: K stays un-rotated, exact.py:38-45)."""
    seq = x_normed.shape[0]
    pos = np.arange(seq) if positions is None else np.asarray(positions)
    if fk is None:
        dk = np.zeros((seq, n_kv, hd), F32)
    else:
        dk = lora_apply(x_normed, *fk).reshape(seq, n_kv, hd)
        if rope is not None:
            if pos.size and int(pos.max()) >= rope[0].shape[0]:
                raise ValueError(f"seq_len {int(pos.max()) + 1} exceeds RoPE cache {rope[0].shape[0]}")
            dk = apply_rope(dk, rope[0], rope[1], pos)
    dv = np.zeros((seq, n_kv, hd), F32) if fv is None else lora_apply(x_normed, *fv).reshape(seq, n_kv, hd)
    return dk.astype(F32), dv.astype(F32)


def page_view(cache: np.ndarray, kv_dim: int = 0) -> np.ndarray:
    if cache.ndim == 4:
        return cache
    if cache.ndim == 5 and cache.shape[0] == 2:
        return cache[kv_dim]
    if cache.ndim == 5 and cache.shape[1] == 2:
        return cache[:, kv_dim]
    raise ValueError(f"unsupported paged KV layout {tuple(cache.shape)}")


def _to_f32(pages: np.ndarray, kind: str) -> np.ndarray:
    if kind == "bf16":
        return bf16_bits_to_f32(pages)
    return pages.astype(F32)


def _from_f32(v: np.ndarray, kind: str) -> np.ndarray:
    if kind == "bf16":
        return f32_to_bf16_bits(v)
    if kind == "f16":
        return v.astype(np.float16)
    return v.astype(F32)


def scatter_into_paged(delta: np.ndarray, cache: np.ndarray, block_table, block_size: int, *,
                       kv_dim: int = 0, kind: str = "f32") -> None:
    """In place: ``pages[bid, :span] = round(fp32(pages) + fp32(delta))``.

    ``kind`` names the page storage: "f32", "f16" (numpy float16) or "bf16" (uint16 bits).
    """
    seq = delta.shape[0]
    need = (seq + block_size - 1) // block_size
    if len(block_table) < need:
        raise ValueError("block_table shorter than prefix")
    pages = page_view(cache, kv_dim)
    for i, bid in enumerate(list(block_table)[:need]):
        start = i * block_size
        end = min(start + block_size, seq)
        span = end - start
        cur = _to_f32(pages[bid, :span], kind)
        pages[bid, :span] = _from_f32(cur + delta[start:end].astype(F32), kind)


def gather_from_paged(cache: np.ndarray, block_table, seq_len: int, block_size: int, *,
                      kv_dim: int = 0) -> np.ndarray:
    pages = page_view(cache, kv_dim)
    out = np.zeros((seq_len,) + pages.shape[2:], dtype=pages.dtype)
    need = (seq_len + block_size - 1) // block_size
    for i, bid in enumerate(list(block_table)[:need]):
        start = i * block_size
        end = min(start + block_size, seq_len)
        out[start:end] = pages[bid, : end - start]
    return out


def dequant_x(x: np.ndarray, x_dtype: str, scale: np.ndarray | None) -> np.ndarray:
    """Stored activations -> fp32: e4m3 bits (uint8) or float16, times a per-row scale."""
    v = e4m3_bits_to_f32(x) if x_dtype == "e4m3" else x.astype(F32)
    if scale is not None:
        v *= scale.astype(F32)[:, None]
    return v


def exact_patch_paged(*, x: np.ndarray, x_dtype: str, x_scale: np.ndarray | None,
                      norm_w: np.ndarray | None, eps: float, factors: list,
                      cu_seqlens: np.ndarray, block_tables: np.ndarray, k_pages: list,
                      v_pages: list, n_kv: int, hd: int, rope=None, kind: str = "bf16",
                      accumulate: bool = True) -> None:
    """Batched exact patch, in place on ``k_pages[l]`` / ``v_pages[l]``
    (``[num_blocks, block_size, n_kv, hd]``).  ``x`` is ``[L, rows, d]``;
    ``factors[l] = (fk, fv)`` as in :func:`exact_kv_delta`; ``norm_w`` ``[L, d]`` or None
    (X already normalised)."""
    n_layers = x.shape[0]
    bs = k_pages[0].shape[1]
    for l in range(n_layers):
        fk, fv = factors[l]
        for b in range(len(cu_seqlens) - 1):
            r0, r1 = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
            if r1 == r0:
                continue
            xs = None if x_scale is None else x_scale[l, r0:r1]
            xv = dequant_x(x[l, r0:r1], x_dtype, xs)
            if norm_w is not None:
                xv = rmsnorm(xv, norm_w[l], eps)
            dk, dv = exact_kv_delta(xv, fk, fv, n_kv, hd, rope)
            table = block_tables[b]
            if accumulate:
                scatter_into_paged(dk, k_pages[l], table, bs, kind=kind)
                scatter_into_paged(dv, v_pages[l], table, bs, kind=kind)
            else:
                for src, pg in ((dk, k_pages[l]), (dv, v_pages[l])):
                    seq = src.shape[0]
                    for i in range(seq):
                        pg[table[i // bs], i % bs] = _from_f32(src[i], kind)
