// Host build of the device numerics (exactattention_b200/csrc/ea_numerics.h), exported with C
// linkage so the CPU tests can compare each helper with the exact oracle. Test-only.
#include "../../exactattention_b200/csrc/ea_numerics.h"

using namespace ea;

static const uint64_t TA64[256] = EA_EXP2_TA64_INIT;
static const uint64_t TB64[256] = EA_EXP2_TB64_INIT;
static const uint64_t TA128[512] = EA_EXP2_TA128_INIT;
static const uint64_t TB128[512] = EA_EXP2_TB128_INIT;

extern "C" {

uint64_t probe_exp2_q63(uint64_t F) { return exp2_q63(F, TA64, TB64); }

void probe_exp2_q127(uint64_t F, uint64_t* hi, uint64_t* lo) {
  u128 y = exp2_q127(F, TA128, TB128);
  *hi = (uint64_t)(y >> 64);
  *lo = (uint64_t)y;
}

// t given as (neg, q, qe); returns status, writes M, E
int probe_weight(int neg, uint64_t q, int qe, int wide, uint32_t* M, int64_t* E) {
  Rnd t = rnd_zero();
  t.neg = neg; t.q = q; t.qe = qe;
  return wide ? weight_from_logit_wide(t, TA128, TB128, *M, *E) : weight_from_logit(t, TA64, TB64, *M, *E);
}

// RN of a/b 2^sh: returns output bits (fp32 or bf16), *ovf
uint32_t probe_round_ratio64(uint64_t a, uint64_t b, int sh, int neg, int fp32, int* ovf) {
  Rnd r = fp32 ? round_ratio64(a, b, sh, neg, FP32_P, FP32_QMIN, FP32_EMAX)
               : round_ratio64(a, b, sh, neg, BF16_P, BF16_QMIN, BF16_EMAX);
  *ovf = r.ovf;
  return fp32 ? rnd_to_f32_bits(r) : rnd_to_bf16_bits(r);
}

// RN of the u128 (hi, lo) * 2^E to fp32 bits
uint32_t probe_round_u128(uint64_t hi, uint64_t lo, int E, int neg, int sticky, int* ovf) {
  Rnd r = round_u128(((u128)hi << 64) | lo, E, neg, FP32_P, FP32_QMIN, FP32_EMAX, sticky != 0);
  *ovf = r.ovf;
  return rnd_to_f32_bits(r);
}

int probe_logit_interval(int64_t acc, uint64_t err, int sexp, uint32_t alpha_bits, uint32_t* t_bits) {
  int32_t am, ae;
  decode_fp32(alpha_bits, am, ae);
  Rnd t = rnd_zero();
  int s = logit_from_interval(acc, err, sexp, am, ae, t);
  *t_bits = rnd_to_f32_bits(t);
  return s;
}

int probe_logit_exact64(int64_t acc, int sexp, uint32_t alpha_bits, uint32_t* t_bits) {
  int32_t am, ae;
  decode_fp32(alpha_bits, am, ae);
  Rnd t = rnd_zero();
  int s = logit_exact64(acc, sexp, am, ae, t);
  *t_bits = rnd_to_f32_bits(t);
  return s;
}

int probe_logit_i128(int64_t hi, uint64_t lo, int E, uint32_t alpha_bits, uint32_t* t_bits) {
  int32_t am, ae;
  decode_fp32(alpha_bits, am, ae);
  Rnd t = rnd_zero();
  i128 S = (i128)(((u128)(uint64_t)hi << 64) | lo);
  int s = logit_i128(S, E, am, ae, t);
  *t_bits = rnd_to_f32_bits(t);
  return s;
}

// exact logit of a q row and a k row of d bf16 values
int probe_logit_exact(const uint16_t* q, const uint16_t* k, int d, uint32_t alpha_bits, uint32_t* t_bits) {
  int32_t am, ae;
  decode_fp32(alpha_bits, am, ae);
  ExactScore s;
  score_clear(s);
  for (int i = 0; i < d; ++i) {
    int32_t qm, qe, km, ke;
    decode_bf16(q[i], qm, qe);
    decode_bf16(k[i], km, ke);
    if (qm && km) score_add(s, qm * km, qe + ke);
  }
  Rnd t = rnd_zero();
  int st = logit_exact(s, am, ae, t);
  *t_bits = rnd_to_f32_bits(t);
  return st;
}

int probe_certify_ratio(int64_t N, uint64_t Nerr, int64_t nunit, int64_t Z, uint64_t Zerr, int64_t zunit, int fp32,
                        uint32_t* bits) {
  Rnd r = rnd_zero();
  bool ok = fp32 ? certify_ratio(N, Nerr, nunit, Z, Zerr, zunit, FP32_P, FP32_QMIN, FP32_EMAX, r)
                 : certify_ratio(N, Nerr, nunit, Z, Zerr, zunit, BF16_P, BF16_QMIN, BF16_EMAX, r);
  *bits = fp32 ? rnd_to_f32_bits(r) : rnd_to_bf16_bits(r);
  return ok ? 1 : 0;
}

void probe_rescale(int64_t* acc, uint64_t* err, int s) { rescale(*acc, *err, s); }

}  // extern "C"
