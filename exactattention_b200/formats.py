"""Host-side helpers of the public API: the domain-error type, bf16 bit conversions for test
inputs, and the default logit scale.

Same names and behaviour as the reference's src/exactattn/formats.py:16-18, 160-181 and
reference.py:164-173.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np


class ExactAttentionDomainError(ValueError):
    """An input is outside the spec's domain (NaN/inf, or an infinite intermediate)."""


def float_to_bf16_bits(x) -> np.ndarray:
    """RN-even conversion of float32-castable values to bf16 bit patterns (uint16), through
    float32 (formats.py:160-176). For making test inputs only."""
    f = np.asarray(x, dtype=np.float32)
    if not np.all(np.isfinite(f)):
        raise ExactAttentionDomainError("non-finite value")
    u = f.view(np.uint32).astype(np.uint64)
    out = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    if np.any((out & 0x7F80) == 0x7F80):
        raise ExactAttentionDomainError("bf16 overflow when generating input")
    return out


def bf16_bits_to_float32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _ln2_bounds(w: int) -> tuple[int, int]:
    """lo <= ln(2) 2^w <= hi from ln 2 = sum_k 2 / ((2k+1) 3^(2k+1)), floors counted."""
    g = w + 16
    s = n = k = 0
    while True:
        t = (2 << g) // ((2 * k + 1) * 3 ** (2 * k + 1))
        if t == 0:
            break
        s += t
        n += 1
        k += 1
    return s >> 16, ((s + n + 2) >> 16) + 1


def _rn_fp32_ratio(num: int, den: int) -> tuple[int, int]:
    """RN-even of num/den > 0 into fp32 (normal range): (m, e)."""
    k = num.bit_length() - den.bit_length()
    if (num << max(0, -k)) < (den << max(0, k)):
        k -= 1
    qe = k - 23
    q, r = divmod(num << -qe, den) if qe < 0 else divmod(num, den << qe)
    d2 = den if qe < 0 else den << qe
    if 2 * r > d2 or (2 * r == d2 and q & 1):
        q += 1
    if q == 1 << 24:
        q, qe = q >> 1, qe + 1
    return q, qe


@lru_cache(maxsize=None)
def default_alpha(d: int) -> np.float32:
    """alpha = RN_fp32(log2(e) / sqrt(d)) = RN_fp32(1 / (ln 2 sqrt d)), decided exactly."""
    w = 96
    while True:
        lo, hi = _ln2_bounds(w)
        s = math.isqrt(d << (2 * w))
        a = _rn_fp32_ratio(1 << (2 * w), hi * (s + 1))
        b = _rn_fp32_ratio(1 << (2 * w), lo * s)
        if a == b:
            return np.float32(a[0] * 2.0 ** a[1])
        w *= 2


@lru_cache(maxsize=None)
def alpha_for(scaling: float) -> np.float32:
    """alpha = RN_fp32(scaling / ln 2) for a model's softmax scaling (a double), decided exactly:
    the base-2 logit multiplier that makes 2^(alpha s) the model's exp(scaling s) up to rounding
    (the reference's scripts/validate_model.py:35-40 `alpha_for`)."""
    num, den = float(scaling).as_integer_ratio()
    if num <= 0:
        raise ValueError("scaling must be positive")
    w = 96
    while True:
        lo, hi = _ln2_bounds(w)
        a = _rn_fp32_ratio(num << w, den * hi)
        b = _rn_fp32_ratio(num << w, den * lo)
        if a == b:
            return np.float32(a[0] * 2.0 ** a[1])
        w *= 2
