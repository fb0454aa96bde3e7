// Wide fixed-point integers for the device fallback tier (tier 3) of certified ExactAttention.
//
// Wide<L> is a carry-save accumulator of L signed 64-bit digits, each standing for 32 bits
// (value = sum_i d[i] 2^(32 i)). Adding a term touches two digits and never propagates a carry,
// so a term costs the same wherever it lands; normalize() propagates carries once, before a
// shift or a read-out. round_ratio_big() is RN-even of a ratio of two wide magnitudes by
// restoring division (p + 2 quotient bits), the wide form of ea_numerics.h round_ratio64.
//
// The reference computes the same quantities with unbounded Python integers
// (src/exactattn/reference.py:111-141); here the window is wide enough that every term of a
// sane row is kept exactly, and any term that is not is counted in a rigorous error bound and
// certified like tier 1 (SPEC section 7).
#pragma once
#include "ea_numerics.h"

namespace ea {

template <int L>
struct Wide {
  int64_t d[L];

  EA_HD void clear() {
    for (int i = 0; i < L; ++i) d[i] = 0;
  }

  // adds floor(v * 2^pos); |v| < 2^33. Returns false if pos is beyond the top digit.
  EA_HD bool add(int64_t v, int64_t pos, uint64_t& err) {
    if (v == 0) return true;
    if (pos < 0) {
      int lost;
      v = floor_shift(v, pos < -64 ? -64 : (int)pos, lost);
      err += (uint64_t)lost;
      pos = 0;
      if (v == 0) return true;
    }
    int limb = (int)(pos >> 5), off = (int)(pos & 31);
    if (limb >= L - 1) return false;
    int64_t x = (int64_t)((uint64_t)v << off);   // |x| < 2^63
    int64_t lo = x & 0xFFFFFFFFll;
    d[limb] += lo;
    d[limb + 1] += (x - lo) >> 32;
    return true;
  }

  EA_HD void normalize() {
    for (int i = 0; i < L - 1; ++i) {
      int64_t c = d[i] >> 32;
      d[i] -= c * 4294967296ll;
      d[i + 1] += c;
    }
  }

  EA_HD bool negative() const { return d[L - 1] < 0; }

  // floor(value / 2^s) for a normalised value; returns whether nonzero bits were dropped.
  EA_HD bool shr(int64_t s) {
    if (s <= 0) return false;
    bool neg = negative();
    if (s >= 32ll * L) {
      bool lost = false;
      for (int i = 0; i < L; ++i) lost |= d[i] != 0;
      for (int i = 0; i < L; ++i) d[i] = 0;
      if (neg) d[0] = -1;  // floor of a negative value is -1 (normalised as top digits)
      if (neg) normalize_minus_one();
      return lost;
    }
    int ls = (int)(s >> 5), bs = (int)(s & 31);
    bool lost = false;
    for (int i = 0; i < ls; ++i) lost |= d[i] != 0;
    if (bs) lost |= (d[ls] & ((1ll << bs) - 1)) != 0;
    // digits are 32-bit two's complement pieces; rebuild as unsigned words with sign fill
    uint32_t w[L];
    for (int i = 0; i < L; ++i) w[i] = (uint32_t)(d[i] & 0xFFFFFFFFll);
    uint32_t fill = neg ? 0xFFFFFFFFu : 0u;
    for (int i = 0; i < L; ++i) {
      int src = i + ls;
      uint32_t lo = src < L ? w[src] : fill;
      uint32_t hi = src + 1 < L ? w[src + 1] : fill;
      uint32_t out = bs ? (uint32_t)((((uint64_t)hi << 32) | lo) >> bs) : lo;
      d[i] = (int64_t)out;
    }
    // restore the signed top digit
    d[L - 1] = (int64_t)(int32_t)(uint32_t)d[L - 1];
    return lost;
  }

  EA_HD void normalize_minus_one() {
    for (int i = 0; i < L - 1; ++i) d[i] = 0xFFFFFFFFll;
    d[L - 1] = -1;
  }

  // magnitude as L + 1 unsigned 32-bit words (normalised input); returns the sign
  EA_HD bool magnitude(uint32_t* out) const {
    bool neg = negative();
    uint64_t carry = 1;
    for (int i = 0; i < L; ++i) {
      uint32_t w = (uint32_t)(d[i] & 0xFFFFFFFFll);
      if (neg) {
        uint64_t x = (uint64_t)(uint32_t)~w + carry;
        out[i] = (uint32_t)x;
        carry = x >> 32;
      } else {
        out[i] = w;
      }
    }
    out[L] = 0;
    return neg;
  }
};

// ---------------------------------------------------------------------------
// unsigned multi-word helpers (little-endian 32-bit words)
// ---------------------------------------------------------------------------
EA_HD int big_bitlen(const uint32_t* a, int n) {
  for (int i = n - 1; i >= 0; --i)
    if (a[i]) return 32 * i + bitlen64(a[i]);
  return 0;
}
EA_HD int big_cmp(const uint32_t* a, const uint32_t* b, int n) {
  for (int i = n - 1; i >= 0; --i)
    if (a[i] != b[i]) return a[i] < b[i] ? -1 : 1;
  return 0;
}
EA_HD void big_shl(const uint32_t* a, int na, int s, uint32_t* out, int n) {  // out = a << s
  int ls = s >> 5, bs = s & 31;
  for (int i = 0; i < n; ++i) {
    int src = i - ls;
    uint32_t lo = (src >= 0 && src < na) ? a[src] : 0u;
    uint32_t lo1 = (src - 1 >= 0 && src - 1 < na) ? a[src - 1] : 0u;
    out[i] = bs ? (uint32_t)((lo << bs) | (lo1 >> (32 - bs))) : lo;
  }
}
EA_HD void big_shr1(uint32_t* a, int n) {
  for (int i = 0; i < n; ++i) a[i] = (a[i] >> 1) | (i + 1 < n ? (a[i + 1] << 31) : 0u);
}
EA_HD void big_sub(uint32_t* a, const uint32_t* b, int n) {  // a -= b, a >= b
  int64_t borrow = 0;
  for (int i = 0; i < n; ++i) {
    int64_t x = (int64_t)a[i] - (int64_t)b[i] - borrow;
    borrow = x < 0;
    a[i] = (uint32_t)(x + (borrow ? 4294967296ll : 0));
  }
}
EA_HD void big_add_u64(uint32_t* a, int n, uint64_t v) {
  uint64_t carry = v;
  for (int i = 0; i < n && carry; ++i) {
    uint64_t x = (uint64_t)a[i] + (carry & 0xFFFFFFFFull);
    a[i] = (uint32_t)x;
    carry = (carry >> 32) + (x >> 32);
  }
}

// RN of (a / b) * 2^sh into (p, qmin, emax); a, b are n-word magnitudes (b > 0), and CAP >= n + 3.
template <int CAP>
EA_HD Rnd round_ratio_big(const uint32_t* a, const uint32_t* b, int n, int64_t sh, int neg, int p, int qmin,
                          int emax) {
  Rnd r = rnd_zero();
  r.neg = neg;
  int bla = big_bitlen(a, n), blb = big_bitlen(b, n);
  if (bla == 0 || blb == 0) return r;
  int k = bla - blb;
  uint32_t t1[CAP], t2[CAP];
  if (k >= 0) {
    big_shl(b, n, k, t2, CAP);
    big_shl(a, n, 0, t1, CAP);
  } else {
    big_shl(a, n, -k, t1, CAP);
    big_shl(b, n, 0, t2, CAP);
  }
  if (big_cmp(t1, t2, CAP) < 0) --k;   // 2^k <= a/b < 2^(k+1)
  int64_t K = (int64_t)k + sh;
  if (K < qmin - 1) return r;
  int64_t qe = K - (p - 1);
  if (qe < qmin) qe = qmin;
  int64_t s2 = sh - qe;                // Q = floor(a 2^s2 / b) < 2^p
  uint32_t A[CAP], B[CAP];
  big_shl(a, n, s2 > 0 ? (int)s2 : 0, A, CAP);
  big_shl(b, n, s2 < 0 ? (int)(-s2) : 0, B, CAP);
  uint32_t Bs[CAP];
  big_shl(B, CAP, p + 1, Bs, CAP);
  uint64_t q = 0;
  for (int i = p + 1; i >= 0; --i) {
    if (big_cmp(A, Bs, CAP) >= 0) {
      big_sub(A, Bs, CAP);
      q |= 1ull << i;
    }
    big_shr1(Bs, CAP);
  }
  // remainder A < B: round up if 2A > B, or 2A == B and q is odd
  uint32_t A2[CAP];
  big_shl(A, CAP, 1, A2, CAP);
  int c = big_cmp(A2, B, CAP);
  if (c > 0 || (c == 0 && (q & 1))) ++q;
  if (q == (1ull << p)) {
    q >>= 1;
    ++qe;
  }
  if (q == 0) return r;
  r.q = q;
  r.qe = (int32_t)qe;
  if (qe + bitlen64(q) - 1 > emax) r.ovf = 1;
  return r;
}

}  // namespace ea
