"""CPU oracle: KIVI per-group quantise / dequantise (TEST INFRASTRUCTURE ONLY).

numpy restatement of ``baselines/kivi_cache.py:44-78`` (lzbaclz/HALO) with the
reference's rounding made explicit: every torch op on an fp16 / bf16 tensor
rounds its exact result once to that type, so each step below is a float32
operation (exact or correctly rounded, and float32 carries enough bits that
the second rounding is innocuous) followed by one round-to-nearest-even into
the storage type.  Values travel as float32 arrays holding exactly
representable fp16 / bf16 numbers.  Cross-checked against the plain-C
restatement ``oracle/kivi_ref.c``.
"""
from __future__ import annotations

import numpy as np

from oracle.scorer import bf16_bits_to_f32, f32_to_bf16_bits


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to fp16 / bf16 (nearest-even), return float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "f32":
        return x
    raise ValueError(dtype)


def quantize_per_group(x: np.ndarray, *, bits: int, group_size: int, dtype: str,
                       unsigned_codes: bool = False):
    """Quantise along the last axis in groups of ``group_size``.

    Follows ``baselines/kivi_cache.py:44-69``: ``x_min/x_max`` per group
    (:64-65); ``scale = (x_max - x_min).clamp_min(1e-8) / qmax`` (:66) with the
    scalar ``1e-8`` first cast to the tensor dtype (fp16 -> 0); ``zero = x_min``
    (:67); ``q = ((x - zero) / scale).round().clamp(0, qmax).to(int8)`` (:68),
    where ``round`` is half-to-even and a NaN quotient (0/0 for a constant
    group) becomes code 0 as torch's int8 cast gives it.

    ``x``: float32 array of fp16/bf16 values, last dim divisible by
    ``group_size``.  The reference casts codes with ``.to(torch.int8)``, so
    8-bit codes 128..255 wrap negative there; ``unsigned_codes=True`` keeps
    them as uint8 0..255 (what a byte-packed store holds).  Returns ``(codes int8 (..., G, gs), scale (..., G, 1),
    zero (..., G, 1))`` with scale/zero as float32 values of ``dtype``.
    """
    qmax = (1 << bits) - 1
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    n = shape[-1]
    assert n % group_size == 0
    xg = x.reshape(*shape[:-1], n // group_size, group_size)
    x_min = xg.min(axis=-1, keepdims=True)
    x_max = xg.max(axis=-1, keepdims=True)
    eps = round_to(np.float32(1e-8), dtype)
    d = round_to(x_max - x_min, dtype)
    d = np.maximum(d, eps)
    scale = round_to(d / np.float32(qmax), dtype)
    zero = x_min
    t = round_to(xg - zero, dtype)
    with np.errstate(divide="ignore", invalid="ignore"):
        u = round_to(t / scale, dtype)
    r = np.rint(u)
    codes = np.where(np.isnan(r), 0.0, np.clip(r, 0, qmax))
    codes = codes.astype(np.uint8) if unsigned_codes else codes.astype(np.int16).astype(np.int8)
    return codes, scale, zero


def dequantize_per_group(codes: np.ndarray, scale: np.ndarray, zero: np.ndarray,
                         *, dtype: str) -> np.ndarray:
    """``x = q.float() * scale.float() + zero.float()`` then one rounding to
    ``dtype``: a float32 multiply and a separate float32 add (no fused
    multiply-add), ``baselines/kivi_cache.py:72-78``.  Returns float32 values
    of ``dtype`` with the group axes flattened."""
    with np.errstate(invalid="ignore", over="ignore"):
        x = codes.astype(np.float32) * scale.astype(np.float32)   # inf scale -> NaN, as torch
        x = (x + zero.astype(np.float32)).astype(np.float32)
    x = round_to(x, dtype)
    return x.reshape(*codes.shape[:-2], codes.shape[-2] * codes.shape[-1])


_POS2 = 16 * (np.arange(16) & 1) + 2 * (np.arange(16) >> 1)   # bit of code e in its word


def pack_codes_2bit(codes: np.ndarray) -> np.ndarray:
    """Pack codes 0..3 of each row (flattened last two axes) into the device
    layout: 16 codes per little-endian 32-bit word, code ``i`` in word
    ``i // 16`` at bit ``16 * (e & 1) + 2 * (e >> 1)``, ``e = i % 16``."""
    c = codes.reshape(*codes.shape[:-2], -1).astype(np.uint32)
    n = c.shape[-1]
    assert n % 16 == 0
    c = c.reshape(*c.shape[:-1], n // 16, 16)              # (..., word, e)
    word = np.bitwise_or.reduce(c << _POS2.astype(np.uint32), axis=-1).astype("<u4")
    return word.view(np.uint8).reshape(*c.shape[:-2], n // 4)


def unpack_codes_2bit(packed: np.ndarray, group_size: int) -> np.ndarray:
    """Inverse of :func:`pack_codes_2bit`, back to ``(..., G, group_size)``."""
    p = np.ascontiguousarray(packed.astype(np.uint8))
    nb = p.shape[-1]
    w = p.reshape(*p.shape[:-1], nb // 4, 4).view("<u4")   # (..., word, 1)
    c = (w >> _POS2.astype(np.uint32)) & 3                 # (..., word, e)
    c = c.reshape(*p.shape[:-1], nb * 4)
    return c.reshape(*c.shape[:-1], c.shape[-1] // group_size, group_size).astype(np.int8)


__all__ = ["round_to", "quantize_per_group", "dequantize_per_group",
           "pack_codes_2bit", "unpack_codes_2bit"]
