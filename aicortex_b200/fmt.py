"""Host-side (numpy) views of the packed int4 format, for inspection and tests.

A group is 32 signed 4-bit codes in four little-endian u32 words (code i in
word i >> 3 at bits 4 * (i & 7)) plus one int8 exponent s; the value of code q
is q * max(2^s / 7, 2^-13) (reference kernels.h:56-85).
"""
from __future__ import annotations

import numpy as np

EPS = np.float32(1.0 / 8192.0)


def unit(s: np.ndarray) -> np.ndarray:
    """Dequantisation factor max(2^s * fl(1/7), 2^-13) in float32."""
    s = np.asarray(s, dtype=np.int8).astype(np.float32)
    return np.maximum(np.ldexp(np.float32(1.0), s.astype(np.int32)).astype(np.float32) * np.float32(1.0 / 7.0),
                      EPS).astype(np.float32)


def codes(words: np.ndarray) -> np.ndarray:
    """Signed codes [..., 8 * W] from packed words [..., W] (any 32-bit dtype)."""
    w = np.ascontiguousarray(words).view(np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    nib = ((w[..., None] >> shifts) & 0xF).astype(np.int8)
    nib = np.where(nib >= 8, nib - 16, nib).astype(np.int8)
    return nib.reshape(*w.shape[:-1], w.shape[-1] * 8)


def dequant(words: np.ndarray, exps: np.ndarray) -> np.ndarray:
    """float32 values [..., C] from words [..., C/8] and exponents [..., C/32]."""
    q = codes(words).astype(np.float32)
    u = np.repeat(unit(exps), 32, axis=-1)
    return (q * u).astype(np.float32)
