// Certified binary64 fast paths of the two per-pair roundings (device only):
//   logit   t = RN32(alpha * s) for an exactly known integer score s = acc * 2^sexp
//   weight  w = RN24(2^t) for an fp32 logit t
// Each evaluates the real value in binary64 with a proven error bound and returns the rounded
// result only when no rounding midpoint lies within that bound of the computed value; otherwise
// it returns false and the caller takes the exact integer path (logit_exact64 / logit_from_interval,
// weight_from_logit). A certified result therefore equals the exact one: the fast paths change
// how fast the bits are found, never which bits.
//
// Rounding to p bits from binary64 drops 53 - p significand bits. For p = 24 those are the low 29
// bits, all in the low word; their distance from the midpoint 2^28, in units of the binary64 ulp,
// is compared with the bound (MARGIN ulps). Within a binade the rounding is monotone and its
// result only changes at midpoints, so a computed value y with |y - x| <= bound and a distance
// above the bound rounds as x does (also when x lies in the neighbouring binade: the midpoints
// next to a power of two are 2^-25 relative away from it).
#pragma once
#include <stdint.h>

#include "ea_numerics.h"
#include "exp2_tables.h"

namespace ea {
namespace f64 {

static __device__ const uint64_t g_exp2_d64[256] = EA_EXP2_D64_INIT;

constexpr int MARGIN = 4;  // ulps; both error bounds below are under 2.1 ulps

// distance of the dropped 29 bits (low word `lo`) from their midpoint, signed
__device__ __forceinline__ int32_t mid_dist29(uint32_t lo) { return (int32_t)(lo & 0x1FFFFFFFu) - 0x10000000; }
__device__ __forceinline__ bool clear_of_mid(int32_t d) { return d > MARGIN || d < -MARGIN; }

// The alpha of a launch as a binary64 (am exact: |am| < 2^24).
__device__ __forceinline__ double alpha_mantissa(int32_t am) { return (double)am; }

// t = RN32(am 2^ae * acc 2^sexp) as fp32 bits, for a normal fp32 result.
//   x = RN64(RN64(acc) * am) * 2^(ae + sexp): two roundings of relative size <= 2^-53 each, so
//   |x - t_exact| <= (2^-52 + 2^-106) |t_exact| < 2.01 ulps of x (the power of two is applied to
//   the exponent field, exactly). am != 0. Straight-line code (selects, no branches), so that a
//   caller's unrolled loop can interleave several evaluations.
__device__ __forceinline__ bool logit_f64(int64_t acc, int sexp, double am_d, int32_t ae, uint32_t& bits) {
  const double x = __dmul_rn(__ll2double_rn(acc), am_d);
  const uint32_t hi = (uint32_t)__double2hiint(x), lo = (uint32_t)__double2loint(x);
  const int32_t e32 = (int32_t)((hi >> 20) & 0x7FFu) - (1023 - 127) + ae + sexp;  // biased fp32 exponent
  const int32_t d = mid_dist29(lo);
  const uint32_t mant = ((hi & 0xFFFFFu) << 3) | (lo >> 29);
  const uint32_t b = (hi & 0x80000000u) | (((uint32_t)e32 << 23) + mant + (d > 0 ? 1u : 0u));
  const bool zero = acc == 0;
  bits = zero ? 0u : b;
  return zero || (e32 >= 1 && e32 <= 253 && clear_of_mid(d));
}

// t = RN32(am 2^ae * (acc 2^sexp + c)) for a score known exactly up to a small correction c (the
// parts of lossy window elements), given as corr with |corr - c| <= corr_err. With u = 2^-53:
//   s = RN(RN(acc) 2^sexp + corr), x = RN(s am): |x - am S| <= |am| (u |acc| 2^sexp + corr_err +
//   u |s|) + u |x| =: B (evaluated with a relative margin); certified when the nearest fp32
//   midpoint lies farther than B from x.
__device__ __forceinline__ bool logit_f64_corr(int64_t acc, int sexp, double corr, double corr_err, double am_d,
                                               int32_t ae, uint32_t& bits) {
  if (sexp < -1000 || sexp > 1000) return false;
  const double u = 1.1102230246251565e-16;  // 2^-53
  const double a = __ll2double_rn(acc);
  const double p2 = __hiloint2double((sexp + 1023) << 20, 0);
  const double s = __fma_rn(a, p2, corr);
  const double x = __dmul_rn(s, am_d);
  const double B = (fabs(am_d) * (u * fabs(a) * p2 + corr_err + u * fabs(s)) + u * fabs(x)) * 1.000001;
  const uint32_t hi = (uint32_t)__double2hiint(x), lo = (uint32_t)__double2loint(x);
  const int32_t ex = (int32_t)((hi >> 20) & 0x7FFu);
  const int32_t e32 = ex - (1023 - 127) + ae;
  // (B far below the fp32 spacing also keeps the interval away from the finer spacing of the
  // binade below a power of two)
  if (s == 0.0 || ex <= 53 || e32 < 1 || e32 > 253 || !(B < fabs(x) * 9.313225746154785e-10)) return false;  // 2^-30
  const double ulp = __hiloint2double((ex - 52) << 20, 0);
  const int32_t d = mid_dist29(lo);
  if (!((double)(d < 0 ? -d : d) * ulp > B)) return false;
  const uint32_t mant = ((hi & 0xFFFFFu) << 3) | (lo >> 29);
  bits = (hi & 0x80000000u) | (((uint32_t)e32 << 23) + mant + (d > 0 ? 1u : 0u));
  return true;
}

// The score interval [acc - err, acc + err] * 2^sexp: certified when both ends are and round to
// the same fp32 value; `differ` reports two certified, different ends (an uncertified logit).
__device__ __forceinline__ bool logit_interval_f64(int64_t acc, uint64_t err, int sexp, double am_d, int32_t ae,
                                                   uint32_t& bits, bool& differ) {
  uint32_t b0, b1;
  differ = false;
  if (!logit_f64(acc - (int64_t)err, sexp, am_d, ae, b0) || !logit_f64(acc + (int64_t)err, sexp, am_d, ae, b1))
    return false;
  differ = b0 != b1;
  bits = b0;
  return !differ;
}

// w = RN24(2^t) = M 2^E (2^23 <= M < 2^24) for the fp32 logit with bits tb, |t| < 2^22.
//   |t| < 2^-27: w = 1 (2^t lies strictly inside the rounding interval of 1).
//   J = floor(256 t), n = floor(t) = J >> 8, j = J mod 256, r = t - J / 256 in [0, 2^-8) (exact:
//   t is a multiple of 2^-50 here). 2^t = 2^n * 2^(j/256) * 2^r with
//   p = r (c1 + r (c2 + r (c3 + r (c4 + r c5)))) ~ 2^r - 1 (Taylor to degree 5; remainder
//   < 2^-60.7) and y = RN(T_j + T_j p), T_j = RN64(2^(j/256)):
//     |p - (2^r - 1)| < 2^-8.53 * 2.74 * 2^-53 + 2^-60.7 < 2^-59.3
//     |y - 2^(j/256 + r)| < 2^-53 * (1 + 2^-8.5) + 2 * 2^-59.3 + 2^-53 < 2.1 * 2^-53 (1.05 ulps)
//   and y < 2 (2^f <= 2^(1 - 2^-50) < 2 - 2^-49.4).
// Straight-line code, as logit_f64.
__device__ __forceinline__ bool weight_f64(uint32_t tb, const uint64_t* tab, uint32_t& M, int32_t& E) {
  const float tf = __uint_as_float(tb);
  const float at = fabsf(tf);
  const bool in_range = at < 4194304.0f;            // |t| < 2^22 (false for NaN)
  const bool one = at < 7.450580596923828125e-9f;   // |t| < 2^-27: w = 1
  const double t = (double)(in_range ? tf : 0.0f);
  constexpr double K = 6755399441055744.0;  // 1.5 * 2^52: its low word is zero
  const double u = __fma_rd(t, 256.0, K);  // K + floor(256 t), exactly
  const int32_t J = (int32_t)__double2loint(u);
  const double r = __fma_rn(u - K, -0.00390625, t);
  double p = __fma_rn(r, __longlong_as_double((long long)EA_EXP2_C5), __longlong_as_double((long long)EA_EXP2_C4));
  p = __fma_rn(r, p, __longlong_as_double((long long)EA_EXP2_C3));
  p = __fma_rn(r, p, __longlong_as_double((long long)EA_EXP2_C2));
  p = __fma_rn(r, p, __longlong_as_double((long long)EA_EXP2_C1));
  p = __dmul_rn(r, p);
  const double T = __longlong_as_double((long long)tab[J & 255]);
  const double y = __fma_rn(T, p, T);
  const uint32_t hi = (uint32_t)__double2hiint(y), lo = (uint32_t)__double2loint(y);
  const int32_t d = mid_dist29(lo);
  const uint32_t m = ((1u << 23) | ((hi & 0xFFFFFu) << 3) | (lo >> 29)) + (d > 0 ? 1u : 0u);
  const bool carry = m == (1u << 24);
  const int32_t e = (J >> 8) - 23 + (int32_t)((hi >> 20) & 0x7FFu) - 1023 + (carry ? 1 : 0);
  M = one ? (1u << 23) : (carry ? (1u << 23) : m);
  E = one ? -23 : e;
  return in_range && (one || clear_of_mid(d));
}

// RN_p of a binary64 estimate x of a ratio times 2^sh, the result a normal number of the target
// format, given that |x - ratio| stays within 4.01 u |ratio| (u = 2^-53), i.e. a few ulps of x:
// certified when the 53 - p dropped bits of x lie more than 8 ulps from their midpoint.
// 1: certified (out set), -1: the integer division decides.
__device__ __forceinline__ int round_ratio_estimate(double x, int sh, int p, int qmin, int emax, Rnd& out) {
  const uint64_t bits = (uint64_t)__double_as_longlong(x);
  const int K = (int)((bits >> 52) & 0x7FF) - 1023 + sh;  // 2^K <= value < 2^(K + 1), up to the error
  if (K - (p - 1) <= qmin || K >= emax) return -1;
  const int Dr = 53 - p;  // dropped bits (29 for fp32, 45 for bf16)
  const uint64_t mant = bits & ((1ull << 52) - 1);
  const int64_t dropped = (int64_t)(mant & ((1ull << Dr) - 1)), half = (int64_t)1 << (Dr - 1);
  const int64_t d = dropped - half;
  if (d <= 8 && d >= -8) return -1;
  uint64_t q = ((mant >> Dr) | (1ull << (p - 1))) + (d > 0 ? 1u : 0u);
  int qe = K - (p - 1);
  if (q == (1ull << p)) {
    q >>= 1;
    ++qe;
  }
  out.q = q;
  out.qe = qe;
  return 1;
}

// RN_p(a / b * 2^sh) for a < 2^63, 0 < b < 2^63: x = RN(RN(a) / RN(b)) has relative error below
// 3.01 u. 0: certain (a == 0), 1: certified, -1: the integer division decides.
__device__ __forceinline__ int ratio_f64(uint64_t a, uint64_t b, int sh, int neg, int p, int qmin, int emax,
                                         Rnd& out) {
  out = rnd_zero();
  out.neg = neg;
  if (a == 0) return 0;
  return round_ratio_estimate(__ddiv_rn(__ull2double_rn(a), __ull2double_rn(b)), sh, p, qmin, emax, out);
}

// The same from a reciprocal of the divisor shared by many ratios, rb = RN(1 / RN(b)):
// x = RN(RN(a) rb) carries four roundings, relative error below (1 + u)^3 / (1 - u) - 1 < 4.01 u.
__device__ __forceinline__ int ratio_f64_rcp(uint64_t a, double rb, int sh, int neg, int p, int qmin, int emax,
                                             Rnd& out) {
  out = rnd_zero();
  out.neg = neg;
  if (a == 0) return 0;
  return round_ratio_estimate(__dmul_rn(__ull2double_rn(a), rb), sh, p, qmin, emax, out);
}

// RN(1 / RN(b)) for ratio_f64_rcp (b > 0), and 0 for b <= 0 (which the callers never divide by)
__device__ __forceinline__ double recip_f64(int64_t b) {
  return b > 0 ? __drcp_rn(__ull2double_rn((uint64_t)b)) : 0.0;
}

// certify_ratio_lh through ratio_f64: 1 certified (out set), 0 not certifiable (the ends differ),
// -1 the integer evaluation decides.
__device__ __forceinline__ int certify_ratio_f64(int64_t nlo, int64_t nhi, int64_t nunit, int64_t zlo, int64_t zhi,
                                                 int64_t zunit, int p, int qmin, int emax, Rnd& out) {
  if (zlo <= 0 || zhi < zlo || nhi < nlo) return -1;
  const int64_t sh64 = nunit - zunit;
  if (sh64 > 100000 || sh64 < -100000) return -1;
  const int sh = (int)sh64;
  uint64_t ln, ld, hn, hd;
  int lneg, hneg;
  if (nlo >= 0) {
    ln = (uint64_t)nlo; ld = (uint64_t)zhi; hn = (uint64_t)nhi; hd = (uint64_t)zlo; lneg = 0; hneg = 0;
  } else if (nhi <= 0) {
    ln = (uint64_t)(-nlo); ld = (uint64_t)zlo; hn = (uint64_t)(-nhi); hd = (uint64_t)zhi; lneg = 1; hneg = 1;
  } else {
    return -1;  // the interval holds zero: the integer evaluation
  }
  Rnd rl, rh;
  const int cl = ratio_f64(ln, ld, sh, lneg, p, qmin, emax, rl);
  const int ch = ratio_f64(hn, hd, sh, hneg, p, qmin, emax, rh);
  if (cl < 0 || ch < 0) return -1;
  if (!rnd_eq(rl, rh)) return 0;
  out = rl;
  if (out.q == 0) out.neg = 0;
  return 1;
}

// certify_ratio_f64 with the divisors' reciprocals given (rzlo = recip_f64(zlo), rzhi =
// recip_f64(zhi)): a row's channels share one Z interval, so one pair of reciprocals serves all.
__device__ __forceinline__ int certify_ratio_f64_rcp(int64_t nlo, int64_t nhi, int64_t nunit, int64_t zlo, int64_t zhi,
                                                     double rzlo, double rzhi, int64_t zunit, int p, int qmin,
                                                     int emax, Rnd& out) {
  if (zlo <= 0 || zhi < zlo || nhi < nlo) return -1;
  const int64_t sh64 = nunit - zunit;
  if (sh64 > 100000 || sh64 < -100000) return -1;
  const int sh = (int)sh64;
  Rnd rl, rh;
  int cl, ch;
  if (nlo >= 0) {
    cl = ratio_f64_rcp((uint64_t)nlo, rzhi, sh, 0, p, qmin, emax, rl);
    ch = ratio_f64_rcp((uint64_t)nhi, rzlo, sh, 0, p, qmin, emax, rh);
  } else if (nhi <= 0) {
    cl = ratio_f64_rcp((uint64_t)(-nlo), rzlo, sh, 1, p, qmin, emax, rl);
    ch = ratio_f64_rcp((uint64_t)(-nhi), rzhi, sh, 1, p, qmin, emax, rh);
  } else {
    return -1;  // the interval holds zero: the integer evaluation
  }
  if (cl < 0 || ch < 0) return -1;
  if (!rnd_eq(rl, rh)) return 0;
  out = rl;
  if (out.q == 0) out.neg = 0;
  return 1;
}

}  // namespace f64
}  // namespace ea
