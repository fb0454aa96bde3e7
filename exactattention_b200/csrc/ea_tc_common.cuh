// Device helpers shared by the tensor-core kernels (prefill and decode, d = dv = 128): block
// fixed point of bf16 elements, byte-digit packing, exact int64 recombination of digit-group
// accumulators, and the exact-score fallback of one (q row, k row) pair.
#pragma once
#include <stdint.h>

#include "ea_core.cuh"
#include "ea_numerics.h"
#include "ea_tables.cuh"
#include "ea_tcgen05.cuh"

// Optional phase clocks (built with -DEA_PHASE_TIMERS): thread 0 of every CTA accumulates the
// cycles between the barriers that separate the phases of the tile loop into the 16 counters
// g_phase_cycles, which each kernel's translation unit defines in its own namespace.
#ifdef EA_PHASE_TIMERS
// EA_PT_DECL goes before a block-wide barrier at the start of the kernel
#define EA_PT_DECL                                 \
  __shared__ unsigned long long ea_pt_acc[16];     \
  if (threadIdx.x < 16) ea_pt_acc[threadIdx.x] = 0;
#define EA_PT_INIT long long pt_last = clock64();
#define EA_PT(i)                        \
  if (tid == 0) {                       \
    const long long pt_now = clock64(); \
    ea_pt_acc[i] += pt_now - pt_last;   \
    pt_last = pt_now;                   \
  }
#define EA_PT_FLUSH \
  if (tid == 0)     \
    for (int i = 0; i < 16; ++i) atomicAdd(&g_phase_cycles[i], ea_pt_acc[i]);
// the same, kept by thread `who` (a second role of a warp-specialised kernel) in counters 8-15
#define EA_PTW_INIT long long ptw_last = clock64();
#define EA_PTW(who, i)                   \
  if (tid == (who)) {                    \
    const long long pt_now = clock64();  \
    ea_pt_acc[8 + (i)] += pt_now - ptw_last; \
    ptw_last = pt_now;                   \
  }
#define EA_PTW_FLUSH(who) \
  if (tid == (who))       \
    for (int i = 0; i < 8; ++i) atomicAdd(&g_phase_cycles[8 + i], ea_pt_acc[8 + i]);
#else
#define EA_PT_DECL
#define EA_PT_INIT
#define EA_PT(i)
#define EA_PT_FLUSH
#define EA_PTW_INIT
#define EA_PTW(who, i)
#define EA_PTW_FLUSH(who)
#endif

namespace ea {
namespace tcc {

constexpr uint32_t T_UNCERT = 0x7FC00001u;  // pass-1 markers in the logit table (t is never NaN)
constexpr uint32_t T_MASKED = 0x7FC00002u;

__device__ __forceinline__ int32_t lead_of(int32_t m, int32_t e) {  // exponent of |m 2^e|'s leading bit
  return e + bitlen64((uint64_t)(m < 0 ? -m : m)) - 1;
}

// floor(x * 2^s) of an int64 (s may be negative); callers keep left shifts in range
__device__ __forceinline__ int64_t shift_floor(int64_t x, int s) {
  if (s >= 0) return (int64_t)((uint64_t)x << s);
  return s <= -63 ? (x < 0 ? -1 : 0) : (x >> (-s));
}
// ceil(u * 2^s): exact for s >= 0 (callers keep it in range), rounded up otherwise
__device__ __forceinline__ uint64_t scale_ceil(uint64_t u, int s) {
  if (s >= 0) return s >= 63 ? (u ? ~0ull >> 2 : 0) : (u << s);
  int r = -s;
  if (r >= 64) return u != 0;
  return (u >> r) + ((u & ((1ull << r) - 1)) != 0);
}

__device__ __forceinline__ Rnd rnd_from_f32(uint32_t b) {
  Rnd t = rnd_zero();
  int32_t m, e;
  decode_fp32(b, m, e);
  t.q = (uint64_t)(m < 0 ? -m : m);
  t.qe = e;
  t.neg = m < 0;
  if (t.q == 0) t.neg = 0;
  return t;
}

// block fixed point of one bf16 element against lsb, as a two's complement int32
__device__ __forceinline__ int32_t fixq(uint32_t bits, int lsb, int& lost, int& bad) {
  int32_t m, e;
  lost = 0;
  if (!decode_bf16(bits, m, e)) {
    bad = 1;
    return 0;
  }
  if (!m) return 0;
  int32_t mag = m < 0 ? -m : m;
  int sh = e - lsb;
  int32_t f;
  if (sh >= 0) {
    f = mag << sh;
  } else {
    int s = -sh;
    f = s >= 31 ? 0 : (mag >> s);
    lost = (s >= 31) ? 1 : ((f << s) != mag);
  }
  return m < 0 ? -f : f;
}

__device__ __forceinline__ int32_t lead_of_bits(uint32_t mag) {  // lead exponent of a nonzero |bf16|
  int32_t m, e;
  decode_bf16(mag, m, e);
  return lead_of(m, e);
}

// Fixed point of the low / high bf16 of word w at lsb, through fp32: the bf16 is exact in fp32,
// the scale 2^-lsb is exact (lsb in [-126, 126]), and the conversion truncates toward zero as
// fixq does; exact whenever |value| / 2^lsb < 2^31.
__device__ __forceinline__ float scale_of(int lsb) { return __int_as_float((127 - lsb) << 23); }
__device__ __forceinline__ uint32_t fixf_lo(uint32_t w, float sc) {
  return (uint32_t)__float2int_rz(__uint_as_float(w << 16) * sc);
}
__device__ __forceinline__ uint32_t fixf_hi(uint32_t w, float sc) {
  return (uint32_t)__float2int_rz(__uint_as_float(w & 0xFFFF0000u) * sc);
}
// Smallest nonzero magnitude of bf16 halves with one signed 16x2 min per word: a nonzero
// magnitude m (1 .. 0x7FFF) maps to m + 0x7FFF (0x8000 .. 0xFFFE, i.e. -32768 .. -2 as signed
// halves, increasing with m) and zero to 0x7FFF (+32767, larger than every nonzero one); the
// 32-bit add cannot carry between halves. NZ_NONE is the start value and the "all zero" result.
constexpr uint32_t NZ_NONE = 0x7FFF7FFFu;
__device__ __forceinline__ uint32_t nz_key(uint32_t mag2) { return mag2 + 0x7FFF7FFFu; }  // mag2 = w & 0x7FFF7FFF
// the smaller of the two halves' keys, as a signed int (32767: no nonzero magnitude)
__device__ __forceinline__ int32_t nz_key_min(uint32_t k) { return min((int32_t)(int16_t)(k & 0xFFFFu), (int32_t)(int16_t)(k >> 16)); }
// the magnitude a key (< 32767) stands for
__device__ __forceinline__ uint32_t nz_key_mag(int32_t k) { return (uint32_t)(k + 32769); }
// 4 x 4 byte transpose: p_k = bytes k of x0 .. x3
__device__ __forceinline__ void transpose4(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, uint32_t& p0,
                                           uint32_t& p1, uint32_t& p2, uint32_t& p3) {
  const uint32_t a = __byte_perm(x0, x1, 0x5140), b = __byte_perm(x0, x1, 0x7362);
  const uint32_t c = __byte_perm(x2, x3, 0x5140), d = __byte_perm(x2, x3, 0x7362);
  p0 = __byte_perm(a, c, 0x5410);
  p1 = __byte_perm(a, c, 0x7632);
  p2 = __byte_perm(b, d, 0x5410);
  p3 = __byte_perm(b, d, 0x7632);
}

// sum_{g < n} D_g 2^(8g) exactly in int64 for n <= 4 int32 groups (|D_g| < 2^25): a chain of
// 32 x 32 -> 64-bit multiply-adds
template <int n>
__device__ __forceinline__ int64_t recomb(const uint32_t* D) {
  int64_t acc = (int64_t)(int32_t)D[0];
  if (n > 1) acc += (int64_t)(int32_t)D[1] * 256;
  if (n > 2) acc += (int64_t)(int32_t)D[2] * 65536;
  if (n > 3) acc += (int64_t)(int32_t)D[3] * 16777216;
  return acc;
}

// byte p of each of four words, packed into one word (byte permutes)
template <int p>
__device__ __forceinline__ uint32_t pack4(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3) {
  constexpr uint32_t sel = (uint32_t)p | ((uint32_t)(p + 4) << 4);
  return __byte_perm(__byte_perm(x0, x1, sel), __byte_perm(x2, x3, sel), 0x5410);
}

// 16 int32 values -> their byte planes 0 .. NP-1, each as one uint4 (16 bytes)
template <int NP>
__device__ __forceinline__ void planes16(const uint32_t* x, uint4* out) {
  uint32_t w[4][4];  // [plane][word]
#pragma unroll
  for (int c = 0; c < 4; ++c)
    transpose4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3], w[0][c], w[1][c], w[2][c], w[3][c]);
#pragma unroll
  for (int p = 0; p < NP; ++p) out[p] = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
}

// int32 fixed-point value of digit planes at (row, byte k) of an R-row K-major tile
__device__ __forceinline__ int32_t read_fix(const uint8_t* planes, uint32_t plane_bytes, uint32_t row, uint32_t k,
                                            uint32_t R) {
  uint32_t o = tc::kmajor_off(row, k, R);
  uint32_t b0 = planes[o], b1 = planes[o + plane_bytes], b2 = planes[o + 2 * plane_bytes];
  int32_t b3 = (int8_t)planes[o + 3 * plane_bytes];
  return (int32_t)(b0 | (b1 << 8) | (b2 << 16)) + (b3 << 24);
}

static __device__ __noinline__ int logit_bounded(int64_t acc, uint64_t err, int sexp, int32_t am, int32_t ae, Rnd& t) {
  return logit_from_interval(acc, err, sexp, am, ae, t);
}

// The integer paths behind the binary64 fast paths, out of line: rarely taken, they would
// otherwise sit between the hot instructions of the tile loops
static __device__ __noinline__ int logit_exact_ool(int64_t acc, int sexp, int32_t am, int32_t ae, Rnd& t) {
  return logit_exact64(acc, sexp, am, ae, t);
}
static __device__ __noinline__ int weight_ool(const Rnd& t, uint32_t& M, int64_t& E) {
  return weight_from_logit(t, g_ta64, g_tb64, M, E);
}

static __device__ __noinline__ int wide_weight(const Rnd& t, uint32_t& M, int64_t& E) {
  return weight_from_logit_wide(t, g_ta128, g_tb128, M, E);
}

// Exact logit of q row `qrow` and k row `krow`, by the whole warp; every lane returns it.
// Products q_i k_i = m 2^e (|m| < 2^16) summed exactly in a 128-bit window whose unit is 118
// bits below the largest product bound; if some product falls below the window, 576-bit bins.
// (Plain arguments, not the kernel's Prob: taking the parameter struct's address would make every
// thread keep a copy of it in local memory.)
static __device__ __noinline__ int warp_exact_logit(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                    int32_t am, int32_t ae, int64_t qrow, int64_t krow, Rnd& t) {
  const int lane = threadIdx.x & 31;
  int32_t pm[4], pe[4];
  int emax = INT32_MIN;
#pragma unroll
  for (int m4 = 0; m4 < 4; ++m4) {
    const int i = lane + 32 * m4;
    int32_t qm, qe, km, ke;
    decode_bf16(q[qrow * 128 + i], qm, qe);
    decode_bf16(k[krow * 128 + i], km, ke);
    pm[m4] = qm * km;
    pe[m4] = qe + ke;
    if (pm[m4]) emax = max(emax, pe[m4] + 16);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
  if (emax == INT32_MIN) {
    t = rnd_zero();
    return LOGIT_OK;
  }
  const int unit = emax - 118;
  bool below = false;
  i128 s = 0;
#pragma unroll
  for (int m4 = 0; m4 < 4; ++m4) {
    if (!pm[m4]) continue;
    const int sh = pe[m4] - unit;
    if (sh < 0) below = true;
    else s += (i128)pm[m4] << sh;
  }
  int ls;
  if (!__any_sync(0xffffffffu, below)) {
    uint64_t lo = (uint64_t)s;
    int64_t hi = (int64_t)(s >> 64);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const uint64_t lo2 = __shfl_xor_sync(0xffffffffu, lo, o);
      const int64_t hi2 = __shfl_xor_sync(0xffffffffu, hi, o);
      const uint64_t sum = lo + lo2;
      hi = hi + hi2 + (sum < lo ? 1 : 0);
      lo = sum;
    }
    ls = logit_i128((i128)(((u128)(uint64_t)hi << 64) | lo), unit, am, ae, t);
  } else {
    ExactScore sc;
    score_clear(sc);
#pragma unroll
    for (int m4 = 0; m4 < 4; ++m4)
      if (pm[m4]) score_add(sc, pm[m4], pe[m4]);
#pragma unroll
    for (int b = 0; b < SCORE_BINS; ++b)
#pragma unroll
      for (int o = 16; o; o >>= 1) sc.bins[b] += __shfl_xor_sync(0xffffffffu, sc.bins[b], o);
    ls = logit_exact(sc, am, ae, t);
  }
  return ls;
}

}  // namespace tcc
}  // namespace ea
