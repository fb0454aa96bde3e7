// Exact integer numerics of certified ExactAttention, shared by every kernel.
//
// Everything here is integer arithmetic on exact dyadic values, written once for both the
// device and the host (the host build exists only so the tests can check these functions
// against the exact oracle on a machine without a GPU).
//
// Definitions followed (reference repository paths):
//   SPEC steps 1-5 ................. docs/SPEC.md:38-55; domain errors docs/SPEC.md:57-65
//   bf16 decode .................... src/exactattn/formats.py:107-117
//   RN-even with gradual underflow . src/exactattn/formats.py:39-85
//   certified logit interval ....... src/exactattn/certified.py:93-138 (Ziv, SPEC section 7)
//   RN24(2^t) ...................... src/exactattn/exp2.py:49-81 (definition); the integer
//                                    evaluation below is this project's own (Tang's method)
//   partial rescale / merge ........ src/exactattn/certified.py:70-86, 213-246
//   certified final ratio .......... src/exactattn/certified.py:249-297
#pragma once
#include <stdint.h>

#include "exp2_tables.h"

#if defined(__CUDACC__)
#define EA_HD __host__ __device__ __forceinline__
#else
#define EA_HD inline
#endif

namespace ea {

typedef unsigned __int128 u128;
typedef __int128 i128;

// ---------------------------------------------------------------------------
// bit utilities
// ---------------------------------------------------------------------------
EA_HD int clz64(uint64_t x) {  // x != 0
#if defined(__CUDA_ARCH__)
  return __clzll((long long)x);
#else
  return __builtin_clzll(x);
#endif
}
EA_HD int bitlen64(uint64_t x) { return x ? 64 - clz64(x) : 0; }
EA_HD int bitlen128(u128 x) {
  uint64_t hi = (uint64_t)(x >> 64);
  return hi ? 64 + bitlen64(hi) : bitlen64((uint64_t)x);
}
EA_HD uint64_t umulhi64(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
  return __umul64hi(a, b);
#else
  return (uint64_t)(((u128)a * b) >> 64);
#endif
}
EA_HD uint64_t uabs64(int64_t x) { return x < 0 ? (uint64_t)0 - (uint64_t)x : (uint64_t)x; }

// ---------------------------------------------------------------------------
// decoding
// ---------------------------------------------------------------------------
// bf16 bits -> m * 2^e (m signed, |m| < 2^8). False for NaN/inf (exponent field 0xFF).
EA_HD bool decode_bf16(uint32_t b, int32_t& m, int32_t& e) {
  uint32_t ex = (b >> 7) & 0xFFu, fr = b & 0x7Fu;
  int32_t mag = ex ? (int32_t)(fr | 0x80u) : (int32_t)fr;
  m = (b & 0x8000u) ? -mag : mag;
  e = ex ? (int32_t)ex - 134 : -133;
  return ex != 0xFFu;
}
// fp32 bits -> m * 2^e (|m| < 2^24). False for NaN/inf.
EA_HD bool decode_fp32(uint32_t b, int32_t& m, int32_t& e) {
  uint32_t ex = (b >> 23) & 0xFFu, fr = b & 0x7FFFFFu;
  int32_t mag = ex ? (int32_t)(fr | 0x800000u) : (int32_t)fr;
  m = (b & 0x80000000u) ? -mag : mag;
  e = ex ? (int32_t)ex - 150 : -149;
  return ex != 0xFFu;
}

// ---------------------------------------------------------------------------
// RN-even into a binary format
// ---------------------------------------------------------------------------
// A rounded dyadic: value (-1)^neg * q * 2^qe. q == 0 is zero (sign ignored). ovf: the rounded
// magnitude exceeds the format's largest finite value.
struct Rnd {
  uint64_t q;
  int32_t qe;
  int32_t neg;
  int32_t ovf;
};

EA_HD Rnd rnd_zero() { Rnd r; r.q = 0; r.qe = 0; r.neg = 0; r.ovf = 0; return r; }

EA_HD bool rnd_eq(const Rnd& a, const Rnd& b) {
  if (a.ovf || b.ovf) return false;
  if (a.q == 0 && b.q == 0) return true;
  return a.q == b.q && a.qe == b.qe && a.neg == b.neg;
}

// RN-even of A * 2^E into precision p, min quantum exponent qmin, max exponent emax.
// sticky: the exact value has further nonzero bits below A's last bit (only ever set when A
// holds at least p + 2 significant bits, so the rounding position lies inside A).
EA_HD Rnd round_u128(u128 A, int E, int neg, int p, int qmin, int emax, bool sticky = false) {
  Rnd r = rnd_zero();
  r.neg = neg;
  int bl = bitlen128(A);
  if (bl == 0) return r;
  int K = bl - 1 + E;                   // leading-bit exponent
  int qe = K - (p - 1);
  if (qe < qmin) qe = qmin;
  int sh = qe - E;                      // bits of A below the quantum
  uint64_t q;
  if (sh <= 0) {
    q = (uint64_t)(A << (-sh));         // exact; bitlen <= p
  } else if (sh > bl) {
    q = 0;                              // A < 2^(sh-1): below half a quantum
  } else if (sh == bl) {
    u128 half = (u128)1 << (sh - 1);
    q = (A > half || (A == half && sticky)) ? 1 : 0;
  } else {
    u128 qq = A >> sh;
    u128 rem = A - (qq << sh);
    u128 half = (u128)1 << (sh - 1);
    q = (uint64_t)qq;
    if (rem > half || (rem == half && (sticky || (q & 1)))) ++q;
  }
  if (q == ((uint64_t)1 << p)) {
    q >>= 1;
    ++qe;
  }
  if (q == 0) return r;
  r.q = q;
  r.qe = qe;
  if (qe + bitlen64(q) - 1 > emax) r.ovf = 1;
  return r;
}

// round_u128 for A < 2^64, in 64-bit arithmetic only (the fast path of the kernels).
EA_HD Rnd round_u64(uint64_t A, int E, int neg, int p, int qmin, int emax, bool sticky = false) {
  Rnd r = rnd_zero();
  r.neg = neg;
  if (A == 0) return r;
  const int bl = bitlen64(A);
  const int K = bl - 1 + E;
  int qe = K - (p - 1);
  if (qe < qmin) qe = qmin;
  const int sh = qe - E;
  uint64_t q;
  if (sh <= 0) {
    q = A << (-sh);
  } else if (sh > bl) {
    q = 0;
  } else if (sh == bl) {
    const uint64_t half = 1ull << (sh - 1);
    q = (A > half || (A == half && sticky)) ? 1 : 0;
  } else {
    q = A >> sh;
    const uint64_t rem = A & ((1ull << sh) - 1), half = 1ull << (sh - 1);
    if (rem > half || (rem == half && (sticky || (q & 1)))) ++q;
  }
  if (q == (1ull << p)) {
    q >>= 1;
    ++qe;
  }
  if (q == 0) return r;
  r.q = q;
  r.qe = qe;
  if (qe + bitlen64(q) - 1 > emax) r.ovf = 1;
  return r;
}

constexpr int FP32_P = 24, FP32_QMIN = -149, FP32_EMAX = 127;
constexpr int BF16_P = 8, BF16_QMIN = -133, BF16_EMAX = 127;

// bits of a rounded fp32 / bf16 value (zero -> +0)
EA_HD uint32_t rnd_to_f32_bits(const Rnd& r) {
  if (r.q == 0) return 0u;
  uint32_t mag = (uint32_t)((int64_t)(r.qe + 149) << 23) + (uint32_t)r.q;
  return mag | (r.neg ? 0x80000000u : 0u);
}
EA_HD uint32_t rnd_to_bf16_bits(const Rnd& r) {
  if (r.q == 0) return 0u;
  uint32_t mag = (uint32_t)((int64_t)(r.qe + 133) << 7) + (uint32_t)r.q;
  return mag | (r.neg ? 0x8000u : 0u);
}

// ---------------------------------------------------------------------------
// certified logit t = RN32(alpha * s) (SPEC step 2)
// ---------------------------------------------------------------------------
enum { LOGIT_OK = 0, LOGIT_UNCERTIFIED = 1, LOGIT_OVERFLOW = 2 };

// s lies in [acc - err, acc + err] * 2^sexp; alpha = am * 2^ae. |acc| + err < 2^63.
// Certified when both ends round to the same fp32 value. Both ends overflowing with one sign
// means t is infinite: a domain error.
EA_HD int logit_from_interval(int64_t acc, uint64_t err, int sexp, int32_t am, int32_t ae, Rnd& t) {
  if (am == 0) {
    t = rnd_zero();
    return LOGIT_OK;
  }
  uint64_t a = uabs64(am);
  int64_t lo = acc - (int64_t)err, hi = acc + (int64_t)err;
  Rnd rl = round_u128((u128)a * uabs64(lo), ae + sexp, (am < 0) != (lo < 0), FP32_P, FP32_QMIN, FP32_EMAX);
  Rnd rh = err ? round_u128((u128)a * uabs64(hi), ae + sexp, (am < 0) != (hi < 0), FP32_P, FP32_QMIN, FP32_EMAX)
               : rl;
  if (rl.ovf && rh.ovf && rl.neg == rh.neg) return LOGIT_OVERFLOW;
  if (!rnd_eq(rl, rh)) return LOGIT_UNCERTIFIED;
  t = rl;
  if (t.q == 0) t.neg = 0;
  return LOGIT_OK;
}

// Exact product of a 128-bit magnitude and a 64-bit one (at most 192 bits), rounded: when it
// exceeds 128 bits its low 64 bits act only as a sticky bit (the rounding point lies far above
// them, and they are the exact low bits of the product, so nothing carries out of them).
EA_HD Rnd round_mul128(u128 a, uint64_t m, int E, int neg, int p, int qmin, int emax) {
  const u128 lo = (u128)(uint64_t)a * m, hi = (u128)(uint64_t)(a >> 64) * m;
  const u128 mid = (lo >> 64) + (u128)(uint64_t)hi;  // < 2^65
  const uint64_t w0 = (uint64_t)lo, w1 = (uint64_t)mid, w2 = (uint64_t)(hi >> 64) + (uint64_t)(mid >> 64);
  if (w2 == 0) return round_u128(((u128)w1 << 64) | w0, E, neg, p, qmin, emax);
  return round_u128(((u128)w2 << 64) | w1, E + 64, neg, p, qmin, emax, w0 != 0);
}

// t = RN32(alpha * acc * 2^sexp) for an exactly known score (err == 0): the exact product
// |acc| |am| (< 2^87) rounded once. (Dropping low bits of |acc| before the multiplication would
// not be exact: their product with am can carry across the rounding midpoint.)
EA_HD int logit_exact64(int64_t acc, int sexp, int32_t am, int32_t ae, Rnd& t) {
  if (am == 0 || acc == 0) {
    t = rnd_zero();
    return LOGIT_OK;
  }
  t = round_u128((u128)uabs64(acc) * uabs64(am), ae + sexp, (am < 0) != (acc < 0), FP32_P, FP32_QMIN, FP32_EMAX);
  if (t.ovf) return LOGIT_OVERFLOW;
  if (t.q == 0) t.neg = 0;
  return LOGIT_OK;
}

// ---------------------------------------------------------------------------
// weights w = RN24(2^t), unbounded exponent (SPEC step 3)
// ---------------------------------------------------------------------------
// Integer evaluation of Y ~ 2^(F/2^50) * 2^63 for 0 <= F < 2^50 (Tang's table-driven method,
// constants from gen_exp2_tables.py):
//   a = F >> 42, b = (F >> 34) & 255, c = F mod 2^34, r = c / 2^50 < 2^-16
//   2^f = 2^(a/256) * 2^(b/65536) * 2^r,  2^r = 1 + x + x^2/2 + x^3/6 + R4,  x = r ln 2
// Error bound, in units of 2^-63 of Y (every step is a floor of an exact integer product):
//   X  = floor(c * LN2_Q64 / 2^50):       |X - x 2^64|          < 1 + 2^-17
//   X2 = floor(X^2 / 2^64), X3 = floor(X2 X / 2^64): |dX2| < 1.0001, |dX3| < 1.001
//   P  = X + X2/2 + X3/6 (floors):        |P - (2^r - 1) 2^64|  < 3.3   (R4 < 0.012 units)
//   Y0 = floor(TA[a] TB[b] / 2^63):       |Y0 - 2^(a/256 + b/65536) 2^63| < 3.0001
//   Y  = Y0 + floor(Y0 P / 2^64):         |Y - 2^f 2^63| < 3.0001 * 1.00002 + 3.3 + 1 < 7.4
// Y < 2^64 - 2^13 because f <= 1 - 2^-50. EXP2_ERR rounds the bound up.
constexpr uint64_t EXP2_ERR = 8;

EA_HD uint64_t exp2_q63(uint64_t F, const uint64_t* TA, const uint64_t* TB) {
  uint32_t a = (uint32_t)(F >> 42), b = (uint32_t)(F >> 34) & 255u;
  uint64_t c = F & ((1ull << 34) - 1);
  uint64_t xh = umulhi64(c, EA_LN2_Q64), xl = c * EA_LN2_Q64;
  uint64_t X = (xh << 14) | (xl >> 50);
  uint64_t X2 = umulhi64(X, X);
  uint64_t X3 = umulhi64(X2, X);
  uint64_t P = X + (X2 >> 1) + X3 / 6;
  uint64_t ta = TA[a], tb = TB[b];
  uint64_t yh = umulhi64(ta, tb), yl = ta * tb;
  uint64_t Y0 = (yh << 1) | (yl >> 63);
  return Y0 + umulhi64(Y0, P);
}

enum { W_OK = 0, W_RISKY = 1, W_HUGE = 2 };

// Splits an fp32 logit t = (-1)^neg q 2^qe into t = n + F 2^-50 (0 <= F < 2^50).
// Returns W_HUGE when |t| >= 2^30, and n = 0, F = 0 when |t| < 2^-27 (then RN24(2^t) = 1:
// 2^t lies strictly between the midpoints 1 - 2^-25 and 1 + 2^-24 around 1).
EA_HD int split_logit(const Rnd& t, int64_t& n, uint64_t& F) {
  n = 0;
  F = 0;
  if (t.q == 0) return W_OK;
  int lead = t.qe + bitlen64(t.q) - 1;
  if (lead >= 30) return W_HUGE;
  if (lead < -27) return W_OK;
  // fp32 values with lead >= -27 are normal with 24-bit q, so qe >= -50.
  if (t.qe >= 0) {
    int64_t v = (int64_t)(t.q << t.qe);
    n = t.neg ? -v : v;
    return W_OK;
  }
  int k = -t.qe;
  uint64_t ip = t.q >> k, fr = t.q & ((1ull << k) - 1);
  if (!t.neg) {
    n = (int64_t)ip;
    F = fr << (50 - k);
  } else if (fr) {
    n = -(int64_t)ip - 1;
    F = ((1ull << k) - fr) << (50 - k);
  } else {
    n = -(int64_t)ip;
  }
  return W_OK;
}

// w = M * 2^E with 2^23 <= M < 2^24. W_RISKY: Y is too close to a rounding midpoint to certify
// (then M is a guess that a wider evaluation must replace).
EA_HD int weight_from_logit(const Rnd& t, const uint64_t* TA, const uint64_t* TB, uint32_t& M, int64_t& E) {
  int64_t n;
  uint64_t F;
  int k = split_logit(t, n, F);
  if (k == W_HUGE) return W_HUGE;
  E = n - 23;
  if (F == 0) {
    M = 1u << 23;
    return W_OK;
  }
  uint64_t Y = exp2_q63(F, TA, TB);
  uint64_t frac = Y & ((1ull << 40) - 1), half = 1ull << 39;
  uint64_t dist = frac > half ? frac - half : half - frac;
  uint64_t m = (Y >> 40) + ((Y >> 39) & 1);
  if (m == (1ull << 24)) {
    m >>= 1;
    E += 1;
  }
  M = (uint32_t)m;
  return dist <= EXP2_ERR ? W_RISKY : W_OK;
}

// ---- 128-bit evaluation, for weights the 64-bit one cannot certify ----
EA_HD u128 mulhi128(u128 a, u128 b) {  // floor(a b / 2^128)
  uint64_t a1 = (uint64_t)(a >> 64), a0 = (uint64_t)a, b1 = (uint64_t)(b >> 64), b0 = (uint64_t)b;
  u128 p00 = (u128)a0 * b0, p01 = (u128)a0 * b1, p10 = (u128)a1 * b0, p11 = (u128)a1 * b1;
  u128 mid = (p00 >> 64) + (uint64_t)p01 + (uint64_t)p10;   // < 3 * 2^64
  return p11 + (p01 >> 64) + (p10 >> 64) + (mid >> 64);
}

// Y ~ 2^(F/2^50) * 2^127 with |Y - 2^f 2^127| < 2^6 (units of 2^-127): the same reduction with
// 128-bit constants and the Taylor series of 2^r to x^7 (x^8/8! < 2^-143). TA128/TB128 hold
// (hi, lo) word pairs.
EA_HD u128 exp2_q127(uint64_t F, const uint64_t* TA128, const uint64_t* TB128) {
  uint32_t a = (uint32_t)(F >> 42), b = (uint32_t)(F >> 34) & 255u;
  uint64_t c = F & ((1ull << 34) - 1);
  // X = floor(c * LN2_Q128 / 2^50) with LN2 = H 2^64 + L: c H 2^64 is a multiple of 2^50, so
  // X = (c H) 2^14 + floor(c L / 2^50) exactly; X < 2^112.
  u128 cl = (u128)c * EA_LN2_Q128_LO, ch = (u128)c * EA_LN2_Q128_HI;
  u128 X = (ch << 14) + (cl >> 50);
  // P = x + x^2/2! + ... + x^7/7! with term_k = floor(term_{k-1} X / 2^128) / k
  u128 term = X, P = X;
  for (int k = 2; k <= 7; ++k) {
    term = mulhi128(term, X) / (u128)k;
    P += term;
  }
  u128 ta = ((u128)TA128[2 * a] << 64) | TA128[2 * a + 1];
  u128 tb = ((u128)TB128[2 * b] << 64) | TB128[2 * b + 1];
  // Y0 = floor(ta tb / 2^127) = 2 * mulhi + top bit of the low half
  uint64_t a1 = (uint64_t)(ta >> 64), a0 = (uint64_t)ta, b1 = (uint64_t)(tb >> 64), b0 = (uint64_t)tb;
  u128 p00 = (u128)a0 * b0, p01 = (u128)a0 * b1, p10 = (u128)a1 * b0, p11 = (u128)a1 * b1;
  u128 mid = (p00 >> 64) + (uint64_t)p01 + (uint64_t)p10;
  u128 h = p11 + (p01 >> 64) + (p10 >> 64) + (mid >> 64);
  uint64_t lowtop = (uint64_t)mid;  // bits 64..127 of the product
  u128 Y0 = (h << 1) | (lowtop >> 63);
  return Y0 + mulhi128(Y0, P);
}

constexpr uint64_t EXP2_ERR128 = 64;

// As weight_from_logit, from the 128-bit evaluation. W_RISKY here is a 2^-97 event per weight.
EA_HD int weight_from_logit_wide(const Rnd& t, const uint64_t* TA128, const uint64_t* TB128, uint32_t& M,
                                 int64_t& E) {
  int64_t n;
  uint64_t F;
  int k = split_logit(t, n, F);
  if (k == W_HUGE) return W_HUGE;
  E = n - 23;
  if (F == 0) {
    M = 1u << 23;
    return W_OK;
  }
  u128 Y = exp2_q127(F, TA128, TB128);
  u128 mask = ((u128)1 << 104) - 1, half = (u128)1 << 103;
  u128 frac = Y & mask;
  u128 dist = frac > half ? frac - half : half - frac;
  uint64_t m = (uint64_t)(Y >> 104) + (uint64_t)((Y >> 103) & 1);
  if (m == (1ull << 24)) {
    m >>= 1;
    E += 1;
  }
  M = (uint32_t)m;
  return dist <= EXP2_ERR128 ? W_RISKY : W_OK;
}

// ---------------------------------------------------------------------------
// fixed-point partials (SPEC step 4 with a running reference exponent, section 5.2)
// ---------------------------------------------------------------------------
// floor(m * 2^sh); lost = bits were dropped. Callers keep left shifts inside int64.
EA_HD int64_t floor_shift(int64_t m, int sh, int& lost) {
  if (sh >= 0) {
    lost = 0;
    return (int64_t)((uint64_t)m << sh);
  }
  int s = -sh;
  if (s >= 63) {
    lost = m != 0;
    return m < 0 ? -1 : 0;
  }
  int64_t v = m >> s;
  lost = (int64_t)((uint64_t)v << s) != m;
  return v;
}

// [acc, acc + err] re-expressed in units 2^s larger (s >= 0): floor, ceil, + 1 if acc lost bits.
EA_HD void rescale(int64_t& acc, uint64_t& err, int s) {
  if (s <= 0) return;
  int lost;
  acc = floor_shift(acc, -s, lost);
  uint64_t e = s >= 64 ? (err != 0) : ((err >> s) + ((err & ((1ull << s) - 1)) != 0));
  err = e + (uint64_t)lost;
}

EA_HD bool fits63(int64_t acc, uint64_t err) {
  uint64_t a = uabs64(acc);
  return a < (1ull << 62) && err < (1ull << 62);
}

// ---------------------------------------------------------------------------
// certified final rounding o = RN(N / Z) (SPEC step 5)
// ---------------------------------------------------------------------------
// RN of (a / b) * 2^sh into (p, qmin, emax), a >= 0, b > 0 (both < 2^64).
EA_HD Rnd round_ratio64(uint64_t a, uint64_t b, int sh, int neg, int p, int qmin, int emax) {
  Rnd r = rnd_zero();
  r.neg = neg;
  if (a == 0) return r;
  int k = bitlen64(a) - bitlen64(b);
  bool less = k >= 0 ? ((u128)a < ((u128)b << k)) : (((u128)a << (-k)) < (u128)b);
  if (less) --k;                        // 2^k <= a/b < 2^(k+1)
  int K = k + sh;
  if (K < qmin - 1) return r;           // below half the smallest quantum
  int qe = K - (p - 1);
  if (qe < qmin) qe = qmin;
  int s2 = sh - qe;                     // Q = floor(a 2^s2 / b) < 2^p
  u128 num = a, den = b;
  if (s2 >= 0) num <<= s2;              // bitlen <= bitlen(b) + p <= 88
  else den <<= -s2;                     // -s2 <= 64
  u128 Q = num / den, R = num - Q * den;
  uint64_t q = (uint64_t)Q;
  if (R > den - R || (R == den - R && (q & 1))) ++q;
  if (q == ((uint64_t)1 << p)) {
    q >>= 1;
    ++qe;
  }
  if (q == 0) return r;
  r.q = q;
  r.qe = qe;
  if (qe + bitlen64(q) - 1 > emax) r.ovf = 1;
  return r;
}

// Both ends of N/Z for N in [nlo, nhi] * 2^nunit and Z in [zlo, zhi] * 2^zunit (zlo > 0, all
// magnitudes below 2^63). Returns true and the value when both ends round alike
// (certified.py:249-286).
EA_HD bool certify_ratio_lh(int64_t nlo_, int64_t nhi_, int64_t nunit, int64_t zlo_, int64_t zhi_, int64_t zunit,
                            int p, int qmin, int emax, Rnd& out) {
  if (zlo_ <= 0 || zhi_ < zlo_ || nhi_ < nlo_) return false;
  int64_t sh64 = nunit - zunit;
  if (sh64 > 100000 || sh64 < -100000) return false;
  int sh = (int)sh64;
  uint64_t zlo = (uint64_t)zlo_, zhi = (uint64_t)zhi_;
  i128 nlo = (i128)nlo_, nhi = (i128)nhi_;
  uint64_t ln, ld, hn, hd;
  int lneg, hneg;
  if (nlo >= 0) {
    ln = (uint64_t)nlo; ld = zhi; hn = (uint64_t)nhi; hd = zlo; lneg = 0; hneg = 0;
  } else if (nhi <= 0) {
    ln = (uint64_t)(-nlo); ld = zlo; hn = (uint64_t)(-nhi); hd = zhi; lneg = 1; hneg = 1;
  } else {
    ln = (uint64_t)(-nlo); ld = zlo; hn = (uint64_t)nhi; hd = zlo; lneg = 1; hneg = 0;
  }
  Rnd rl = round_ratio64(ln, ld, sh, lneg, p, qmin, emax);
  Rnd rh = round_ratio64(hn, hd, sh, hneg, p, qmin, emax);
  if (!rnd_eq(rl, rh)) return false;
  out = rl;
  if (out.q == 0) out.neg = 0;
  return true;
}

// N in [N, N + Nerr] * 2^nunit and Z in [Z, Z + Zerr] * 2^zunit (Z > 0)
EA_HD bool certify_ratio(int64_t N, uint64_t Nerr, int64_t nunit, int64_t Z, uint64_t Zerr, int64_t zunit,
                         int p, int qmin, int emax, Rnd& out) {
  if (Z <= 0 || Nerr >= (1ull << 62) || Zerr >= (1ull << 62)) return false;
  return certify_ratio_lh(N, N + (int64_t)Nerr, nunit, Z, Z + (int64_t)Zerr, zunit, p, qmin, emax, out);
}

// t = RN32(alpha * S * 2^E) for an exact signed 128-bit S (|S| < 2^126).
EA_HD int logit_i128(i128 S, int E, int32_t am, int32_t ae, Rnd& t) {
  if (am == 0 || S == 0) {
    t = rnd_zero();
    return LOGIT_OK;
  }
  const int neg = (S < 0) != (am < 0);
  const u128 a = S < 0 ? (u128)(-S) : (u128)S;
  t = round_mul128(a, uabs64(am), ae + E, neg, FP32_P, FP32_QMIN, FP32_EMAX);
  if (t.ovf) return LOGIT_OVERFLOW;
  if (t.q == 0) t.neg = 0;
  return LOGIT_OK;
}

// ---------------------------------------------------------------------------
// exact score on the fallback path (SPEC step 1 without any window)
// ---------------------------------------------------------------------------
// Products of decoded bf16 are m * 2^e with |m| < 2^16 and -266 <= e <= 254. Each goes into a
// 32-bit-digit bin at bit e + 266 (carry-save int64 bins, normalised once at the end), so the
// sum is exact for any d <= 65536.
constexpr int SCORE_BINS = 18;           // 576 bits >= 520 + 17 + 16 + sign
constexpr int SCORE_BIAS = 266;

struct ExactScore {
  int64_t bins[SCORE_BINS];
};

EA_HD void score_clear(ExactScore& s) {
  for (int i = 0; i < SCORE_BINS; ++i) s.bins[i] = 0;
}
EA_HD void score_add(ExactScore& s, int32_t m, int32_t e) {
  int pos = e + SCORE_BIAS;
  int b = pos >> 5, off = pos & 31;
  int64_t v = (int64_t)m << off;        // |v| < 2^47
  int64_t lo = v & 0xFFFFFFFFll;        // in [0, 2^32)
  s.bins[b] += lo;
  s.bins[b + 1] += (v - lo) >> 32;      // exact
}
// Normalises to two's complement 32-bit digits (top bin keeps the sign).
EA_HD void score_normalize(ExactScore& s) {
  for (int i = 0; i < SCORE_BINS - 1; ++i) {
    int64_t c = s.bins[i] >> 32;
    s.bins[i] -= c << 32;
    s.bins[i + 1] += c;
  }
}

// t = RN32(alpha * S * 2^-266) for the normalised exact score. LOGIT_OVERFLOW: domain error.
EA_HD int logit_exact(ExactScore& s, int32_t am, int32_t ae, Rnd& t) {
  score_normalize(s);
  int neg = s.bins[SCORE_BINS - 1] < 0;
  uint32_t mag[SCORE_BINS];
  // magnitude digits
  uint64_t carry = 1;
  for (int i = 0; i < SCORE_BINS; ++i) {
    uint32_t d = (uint32_t)(s.bins[i] & 0xFFFFFFFFll);
    if (neg) {
      uint64_t x = (uint64_t)(uint32_t)~d + carry;
      mag[i] = (uint32_t)x;
      carry = x >> 32;
    } else {
      mag[i] = d;
    }
  }
  int top = -1;
  for (int i = SCORE_BINS - 1; i >= 0; --i)
    if (mag[i]) { top = i; break; }
  if (top < 0 || am == 0) {
    t = rnd_zero();
    return LOGIT_OK;
  }
  // the exact product |S| |am| in 32-bit digits (one more digit than S), then its top 64 bits
  // (aligned at the leading bit) with a sticky bit for the exact bits below them
  uint32_t prod[SCORE_BINS + 1];
  const uint64_t am_mag = uabs64(am);
  uint64_t cy = 0;
  for (int i = 0; i <= top; ++i) {
    const uint64_t x = (uint64_t)mag[i] * am_mag + cy;  // < 2^56 + 2^24
    prod[i] = (uint32_t)x;
    cy = x >> 32;
  }
  int ptop = top;
  if (cy) prod[++ptop] = (uint32_t)cy;
  int lb = 31 - (bitlen64(prod[ptop]) - 1);   // leading zeros in the top digit
  uint64_t w2 = (uint64_t)prod[ptop] << 32 | (ptop >= 1 ? prod[ptop - 1] : 0u);
  uint32_t w0 = ptop >= 2 ? prod[ptop - 2] : 0u;
  uint64_t hi64 = lb ? (w2 << lb) | ((uint64_t)w0 >> (32 - lb)) : w2;
  bool sticky = (lb ? (uint32_t)(w0 << lb) != 0u : w0 != 0u);
  for (int i = ptop - 3; i >= 0 && !sticky; --i) sticky = prod[i] != 0u;
  int e_hi = (ptop - 1) * 32 - lb - SCORE_BIAS;  // exponent of hi64's last bit
  t = round_u64(hi64, ae + e_hi, neg != (am < 0), FP32_P, FP32_QMIN, FP32_EMAX, sticky);
  if (t.ovf) return LOGIT_OVERFLOW;
  if (t.q == 0) t.neg = 0;
  return LOGIT_OK;
}

}  // namespace ea
