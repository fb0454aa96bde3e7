"""Exact ExactAttention v0 on the CPU, in plain Python integers.

TEST INFRASTRUCTURE ONLY. The product never imports this module: only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and only as the checker.

This is a restatement of the reference's ground truth (reference repo paths):

  bf16 / fp32 decoding ............ src/exactattn/formats.py:107-131, reference.py:33-44
  RN-even of a rational ........... src/exactattn/formats.py:39-85
  exact score and logit ........... src/exactattn/reference.py:47-79
  RN24(2^t) weight (Ziv loop) ..... src/exactattn/exp2.py:49-81
  exact Z, N and the one rounding . src/exactattn/reference.py:82-143
  batched mask / CSR drivers ...... src/exactattn/reference.py:150-161, cpu.py:62-68
  default_alpha ................... src/exactattn/reference.py:164-173

The exp2 oracle here does not use mpmath (the reference does). It encloses 2^f with integer
interval arithmetic (ln 2 from the atanh series, e^y from its Taylor series with a proven
truncation bound) and doubles the working precision until the enclosure decides the rounding.
2^f is irrational for non-integer dyadic f (SPEC 5.1), so the loop always ends.
"""

from __future__ import annotations

import struct
from functools import lru_cache

import numpy as np


class ExactAttentionDomainError(ValueError):
    """Input outside the spec's domain: NaN/inf, or an fp32 logit that overflows."""


# (precision p, minimum quantum exponent qmin, maximum exponent emax); None = unbounded.
BF16 = (8, -133, 127)
FP32 = (24, -149, 127)
FP24INF = (24, None, None)

# reference.py:30 - the reference refuses weight exponent spreads above this.
MAX_EXPONENT_SPREAD = 1 << 20


# ---------------------------------------------------------------------------
# decoding / encoding (formats.py:107-158)
# ---------------------------------------------------------------------------

def decode_bf16(bits: int) -> tuple[int, int]:
    b = int(bits) & 0xFFFF
    ex = (b >> 7) & 0xFF
    fr = b & 0x7F
    if ex == 0xFF:
        raise ExactAttentionDomainError("bf16 NaN or infinity in input")
    m = fr if ex == 0 else (fr | 0x80)
    e = -133 if ex == 0 else ex - 134
    return (-m if b & 0x8000 else m), e


def decode_bf16_np(bits) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Vectorised decode: (m int64, e int64, bad bool) with value m * 2**e."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.int64)
    ex = (b >> 7) & 0xFF
    fr = b & 0x7F
    m = np.where(ex != 0, fr | 0x80, fr)
    m = np.where((b & 0x8000) != 0, -m, m)
    e = np.where(ex != 0, ex - 134, -133)
    return m, e, ex == 0xFF


def f32_to_bits(x) -> int:
    return struct.unpack("<I", struct.pack("<f", float(np.float32(x))))[0]


def decode_fp32(x) -> tuple[int, int]:
    u = f32_to_bits(x)
    ex = (u >> 23) & 0xFF
    fr = u & 0x7FFFFF
    if ex == 0xFF:
        raise ExactAttentionDomainError("fp32 NaN or infinity in input")
    m = fr if ex == 0 else (fr | 0x800000)
    e = -149 if ex == 0 else ex - 150
    return (-m if u & 0x80000000 else m), e


def encode(m: int, e: int, out: str):
    """Bits (bf16, as int) or value (fp32, as np.float32) of the representable m * 2**e.
    Zero of either sign encodes as +0 (SPEC step 5)."""
    if m == 0:
        return 0 if out == "bf16" else np.float32(0.0)
    x = float(m) * 2.0 ** e                 # exact: |m| < 2^24 and -149 <= e <= 104
    f = np.float32(x)
    assert float(f) == x, "value is not fp32-representable"
    if out == "fp32":
        return f
    u = f32_to_bits(f)
    assert u & 0xFFFF == 0, "value is not bf16-representable"
    return u >> 16


# ---------------------------------------------------------------------------
# RN-even of an exact rational (formats.py:39-85)
# ---------------------------------------------------------------------------

def round_ratio(num: int, den: int, fmt) -> tuple[int, int]:
    """RN-even of num/den into fmt = (p, qmin, emax). Returns (m, e), m signed, |m| < 2**p;
    (0, 0) for zero. Raises ExactAttentionDomainError on overflow past emax."""
    p, qmin, emax = fmt
    if den == 0:
        raise ZeroDivisionError("round_ratio: zero denominator")
    if den < 0:
        num, den = -num, -den
    if num == 0:
        return (0, 0)
    neg = num < 0
    a = -num if neg else num
    k = a.bit_length() - den.bit_length()          # 2^k <= a/den < 2^(k+1) after the fix-up
    if (a << max(0, -k)) < (den << max(0, k)):
        k -= 1
    qe = k - (p - 1)
    if qmin is not None and qe < qmin:
        qe = qmin
    if qe >= 0:
        q, r = divmod(a, den << qe)
        d2 = den << qe
    else:
        q, r = divmod(a << -qe, den)
        d2 = den
    if 2 * r > d2 or (2 * r == d2 and (q & 1)):
        q += 1
    if q == 1 << p:
        q >>= 1
        qe += 1
    if q == 0:
        return (0, 0)
    if emax is not None and qe + q.bit_length() - 1 > emax:
        raise ExactAttentionDomainError("overflow")
    return (-q if neg else q), qe


def round_dyadic(m: int, e: int, fmt) -> tuple[int, int]:
    return round_ratio(m << e, 1, fmt) if e >= 0 else round_ratio(m, 1 << -e, fmt)


# ---------------------------------------------------------------------------
# RN24(2^t) with an unbounded exponent (exp2.py:49-81), integer interval arithmetic
# ---------------------------------------------------------------------------

@lru_cache(maxsize=64)
def _ln2_bounds(w: int) -> tuple[int, int]:
    """(lo, hi) with lo <= ln(2) * 2**w <= hi, from ln 2 = sum_k 2 / ((2k+1) 3^(2k+1))."""
    g = w + 16
    one = 1 << g
    s = 0
    terms = 0
    k = 0
    while True:
        den = (2 * k + 1) * 3 ** (2 * k + 1)
        t = (2 * one) // den                      # floor: error < 1 per term
        if t == 0:
            break
        s += t
        terms += 1
        k += 1
    # dropped tail: sum of terms each < 1 unit, decreasing by a factor 9 -> < 2 units
    lo = s >> 16
    hi = ((s + terms + 2) >> 16) + 1
    return lo, hi


def _exp_floor_sum(y: int, w: int) -> tuple[int, int]:
    """S = sum_i floor-chain(y^i / i!) in units 2**-w for 0 <= y < 2**w (y in units 2**-w).
    Returns (S, K): S <= e^(y/2^w) * 2^w <= S + K*K + 2*K + 2 (floor error <= i on term i,
    and the tail after the first zero term is below twice that term's bound)."""
    one = 1 << w
    s = one
    term = one
    i = 1
    while True:
        term = (term * y) // (i << w)
        if term == 0:
            break
        s += term
        i += 1
    return s, i


def _exp2_frac_bounds(F: int, k: int, w: int) -> tuple[int, int]:
    """(lo, hi) with lo <= 2^(F/2^k) * 2**w <= hi, for 0 < F < 2^k."""
    l_lo, l_hi = _ln2_bounds(w + 8)
    g = w + 8
    y_lo = (F * l_lo) >> k                       # floor(F ln2 / 2^k) in units 2^-g
    y_hi = -((-(F * l_hi)) >> k)                 # ceil
    s_lo, _ = _exp_floor_sum(y_lo, g)
    s_hi, K = _exp_floor_sum(y_hi, g)
    s_hi += K * K + 2 * K + 2
    return s_lo >> 8, -((-s_hi) >> 8)


def split_fp32_dyadic(m: int, e: int) -> tuple[int, int, int]:
    """t = m * 2**e  ->  (n, F, k) with t = n + F / 2**k, 0 <= F < 2**k."""
    if e >= 0:
        return m << e, 0, 0
    k = -e
    n = m >> k                                   # floor
    return n, m - (n << k), k


@lru_cache(maxsize=1 << 18)
def exp2_rn24(tm: int, te: int) -> tuple[int, int]:
    """w = RN_FP24inf(2^t) for the exact dyadic t = tm * 2**te. Returns (M, E), 2^23 <= M < 2^24."""
    n, F, k = split_fp32_dyadic(tm, te)
    if F == 0:
        return 1 << 23, n - 23
    w = 96
    while True:
        lo, hi = _exp2_frac_bounds(F, k, w)      # 2^f * 2^w in [lo, hi], 2^f in (1, 2)
        sh = w - 23
        half = 1 << (sh - 1)
        a = (lo + half) >> sh
        b = (hi + half) >> sh
        if a == b:
            e = n - 23
            if a == 1 << 24:
                a >>= 1
                e += 1
            return a, e
        w *= 2
        if w > 1 << 16:
            raise RuntimeError("exp2 oracle did not converge")


def exp2_rn24_f32(t: float) -> tuple[int, int]:
    m, e = decode_fp32(t)
    return exp2_rn24(m, e)


# ---------------------------------------------------------------------------
# default_alpha (reference.py:164-173): RN_fp32(1 / (ln2 * sqrt(d)))
# ---------------------------------------------------------------------------

def _isqrt(x: int) -> int:
    import math
    return math.isqrt(x)


def default_alpha(d: int) -> np.float32:
    w = 96
    while True:
        l_lo, l_hi = _ln2_bounds(w)
        s_lo = _isqrt(d << (2 * w))
        s_hi = s_lo + 1
        # 1/(ln2 sqrt d) in [2^(2w)/(l_hi s_hi), 2^(2w)/(l_lo s_lo)]
        a = round_ratio(1 << (2 * w), l_hi * s_hi, FP32)
        b = round_ratio(1 << (2 * w), l_lo * s_lo, FP32)
        if a == b:
            return np.float32(a[0] * 2.0 ** a[1])
        w *= 2


# ---------------------------------------------------------------------------
# exact attention (reference.py:47-161)
# ---------------------------------------------------------------------------

def exact_score(qm, qe, km, ke) -> tuple[int, int]:
    """Exact sum_i q_i k_i as (S, E) with value S * 2**E."""
    pm = (np.asarray(qm, dtype=np.int64) * np.asarray(km, dtype=np.int64))
    pe = (np.asarray(qe, dtype=np.int64) + np.asarray(ke, dtype=np.int64))
    nz = pm != 0
    if not nz.any():
        return 0, 0
    pm, pe = pm[nz].tolist(), pe[nz].tolist()
    emin = min(pe)
    s = 0
    for m, e in zip(pm, pe):
        s += m << (e - emin)
    return s, emin


def row_trace(q_bits, k_bits, v_bits, alpha, out: str = "bf16") -> dict:
    """One query row, exactly. Returns every intermediate: s, t (exact dyadics), w, Z, N, out."""
    if out not in ("bf16", "fp32"):
        raise ValueError("out must be 'bf16' or 'fp32'")
    fmt = BF16 if out == "bf16" else FP32
    q_bits = np.asarray(q_bits, dtype=np.uint16).reshape(-1)
    d = q_bits.shape[0]
    k_bits = np.asarray(k_bits, dtype=np.uint16).reshape(-1, d)
    n = k_bits.shape[0]
    v_bits = np.asarray(v_bits, dtype=np.uint16)
    dv = v_bits.shape[-1] if v_bits.ndim == 2 else (v_bits.size // max(n, 1))
    v_bits = v_bits.reshape(n, dv)
    am, ae = decode_fp32(alpha)
    qm, qe, qb = decode_bf16_np(q_bits)
    km, ke, kb = decode_bf16_np(k_bits)
    vm, ve, vb = decode_bf16_np(v_bits)
    if qb.any() or kb.any() or vb.any():
        raise ExactAttentionDomainError("bf16 NaN or infinity in input")
    zero_out = [0] * dv if out == "bf16" else [np.float32(0.0)] * dv
    if n == 0:
        return dict(s=[], t=[], w=[], Z=(0, 0), N=[(0, 0)] * dv, out=zero_out)
    s, t, w = [], [], []
    for j in range(n):
        sj = exact_score(qm, qe, km[j], ke[j])
        s.append(sj)
        if sj[0] == 0 or am == 0:
            tj = (0, 0)
        else:
            tj = round_dyadic(am * sj[0], ae + sj[1], FP32)   # raises on fp32 overflow
        t.append(tj)
        w.append(exp2_rn24(*tj))
    wE = [e for _, e in w]
    emin = min(wE)
    if max(wE) - emin > MAX_EXPONENT_SPREAD:
        raise ExactAttentionDomainError("weight exponent spread exceeds reference limit")
    Z = 0
    for M, E in w:
        Z += M << (E - emin)
    vml, vel = vm.tolist(), ve.tolist()
    N, res = [], []
    for c in range(dv):
        terms = [(w[j][0] * vml[j][c], w[j][1] + vel[j][c]) for j in range(n) if vml[j][c] != 0]
        if not terms:
            N.append((0, 0))
            res.append(zero_out[0])
            continue
        base = min(e for _, e in terms)
        acc = 0
        for m, e in terms:
            acc += m << (e - base)
        N.append((acc, base))
        sh = base - emin
        num, den = (acc << sh, Z) if sh >= 0 else (acc, Z << -sh)
        om, oe = round_ratio(num, den, fmt)
        res.append(encode(om, oe, out))
    return dict(s=s, t=t, w=w, Z=(Z, emin), N=N, out=res)


def attention_row(q_bits, k_bits, v_bits, alpha, out: str = "bf16") -> np.ndarray:
    r = row_trace(q_bits, k_bits, v_bits, alpha, out)["out"]
    return np.array(r, dtype=np.uint16 if out == "bf16" else np.float32)


def attention(q_bits, k_bits, v_bits, alpha, mask=None, out: str = "bf16") -> np.ndarray:
    """q (r, d), k (n, d), v (n, dv) bf16 bits; mask (r, n) bool or None (all keys)."""
    q_bits = np.asarray(q_bits, dtype=np.uint16)
    k_bits = np.asarray(k_bits, dtype=np.uint16)
    v_bits = np.asarray(v_bits, dtype=np.uint16)
    r, dv = q_bits.shape[0], v_bits.shape[1]
    res = np.zeros((r, dv), dtype=np.uint16 if out == "bf16" else np.float32)
    for i in range(r):
        sel = np.arange(k_bits.shape[0]) if mask is None else np.flatnonzero(mask[i])
        res[i] = attention_row(q_bits[i], k_bits[sel], v_bits[sel], alpha, out)
    return res


def attention_csr(q_bits, k_bits, v_bits, alpha, row_ptr, key_idx, out: str = "bf16",
                  rows=None) -> np.ndarray:
    """Row r attends key_idx[row_ptr[r]:row_ptr[r+1]] (any order, cpu.py:62-68 layout).
    `rows` restricts the computation to those row indices (others stay zero)."""
    q_bits = np.asarray(q_bits, dtype=np.uint16)
    dv = np.asarray(v_bits).shape[1]
    res = np.zeros((q_bits.shape[0], dv), dtype=np.uint16 if out == "bf16" else np.float32)
    for i in (range(q_bits.shape[0]) if rows is None else rows):
        sel = np.asarray(key_idx[row_ptr[i]:row_ptr[i + 1]], dtype=np.int64)
        res[i] = attention_row(q_bits[i], k_bits[sel], v_bits[sel], alpha, out)
    return res


def csr_from_mask(mask: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    mask = np.asarray(mask, dtype=bool)
    row_ptr = np.concatenate([[0], np.cumsum(mask.sum(axis=1))]).astype(np.int64)
    key_idx = (np.concatenate([np.flatnonzero(m) for m in mask]).astype(np.int64)
               if mask.size else np.zeros(0, np.int64))
    return row_ptr, key_idx
