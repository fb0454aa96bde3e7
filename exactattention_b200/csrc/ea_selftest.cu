// Self-test of the binary64 fast paths against the exact integer evaluations, on the device.
//
//   mode 0 (weights): logits t taken as consecutive fp32 bit patterns from `seed` (stride
//     `stride`, both signs), restricted to |t| < 2^22; every certified fast weight must equal the
//     integer RN24(2^t) (weight_from_logit, or its 128-bit form when that one is not certain).
//   mode 1 (logits): scores acc (random bit lengths 1..62, both signs), alpha mantissas and score
//     exponents from a splitmix64 stream; every certified fast logit must equal logit_exact64.
//   mode 2 (output ratios): a / b * 2^sh for random a, b < 2^63 of random lengths, rounded to bf16
//     and to fp32; every certified fast ratio must equal round_ratio64.
//   mode 3: the same through the shared-reciprocal form (ratio_f64_rcp).
// out[0] cases checked, out[1] certified by the fast path, out[2] mismatches, out[3] the input of
// one mismatch (the fp32 bits of t, or the case index).
#include <cuda_runtime.h>
#include <stdint.h>

#include "ea_fast64.cuh"
#include "ea_numerics.h"
#include "ea_tables.cuh"
#include "ea_tc_common.cuh"

namespace ea {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ __forceinline__ void tally(unsigned long long* acc, bool certified, bool bad, uint64_t what) {
  const unsigned m = __activemask();
  const unsigned nc = __popc(__ballot_sync(m, certified)), nb = __popc(__ballot_sync(m, bad));
  const int leader = __ffs(m) - 1;
  if ((int)(threadIdx.x & 31) == leader) {
    atomicAdd(acc + 0, (unsigned long long)__popc(m));
    if (nc) atomicAdd(acc + 1, (unsigned long long)nc);
    if (nb) atomicAdd(acc + 2, (unsigned long long)nb);
  }
  if (bad) acc[3] = what;
}

__global__ void selftest_weight_kernel(uint32_t start, uint32_t stride, int64_t n, unsigned long long* acc) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t mag = (uint32_t)((start + (uint64_t)(i >> 1) * stride) % 0x4A800000u);  // |t| < 2^22
    const uint32_t tb = mag | ((uint32_t)(i & 1) << 31);
    uint32_t Mf = 0;
    int32_t Ef = 0;
    const bool cert = f64::weight_f64(tb, f64::g_exp2_d64, Mf, Ef);
    bool bad = false;
    if (cert) {
      const Rnd t = tcc::rnd_from_f32(tb);
      uint32_t M;
      int64_t E;
      int ws = weight_from_logit(t, g_ta64, g_tb64, M, E);
      if (ws == W_RISKY) ws = weight_from_logit_wide(t, g_ta128, g_tb128, M, E);
      bad = ws == W_OK && (M != Mf || E != (int64_t)Ef);
    }
    tally(acc, cert, bad, tb);
  }
}

__global__ void selftest_logit_kernel(uint64_t seed, int64_t n, unsigned long long* acc) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h0 = mix64(seed ^ (uint64_t)i), h1 = mix64(h0), h2 = mix64(h1);
    const int len = 1 + (int)(h0 % 62);
    int64_t a = (int64_t)(h1 >> (64 - len));
    if (h0 & (1ull << 40)) a = -a;
    int32_t am = (int32_t)((h2 & 0x7FFFFFu) | 0x800000u);
    if (h2 & (1ull << 30)) am = -am;
    const int32_t ae = -23 - (int32_t)((h2 >> 32) % 8);
    const int sexp = -60 + (int)((h2 >> 40) % 90);
    uint32_t bf = 0;
    const bool cert = f64::logit_f64(a, sexp, (double)am, ae, bf);
    bool bad = false;
    if (cert) {
      Rnd t = rnd_zero();
      const int ls = logit_exact64(a, sexp, am, ae, t);
      bad = ls != LOGIT_OK || rnd_to_f32_bits(t) != bf;
    }
    tally(acc, cert, bad, (uint64_t)i);
  }
}

__global__ void selftest_ratio_kernel(uint64_t seed, int64_t n, int rcp, unsigned long long* acc) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h0 = mix64(seed ^ (uint64_t)i), h1 = mix64(h0), h2 = mix64(h1), h3 = mix64(h2);
    const uint64_t a = h1 >> (1 + h0 % 63), b = (h2 >> (1 + (h0 >> 8) % 63)) | 1u;
    const int sh = -80 + (int)((h3 >> 8) % 120);
    const int neg = (int)(h3 & 1);
    const bool f32 = (h3 >> 1) & 1;
    const int p = f32 ? FP32_P : BF16_P, qmin = f32 ? FP32_QMIN : BF16_QMIN;
    Rnd rf;
    const int c = rcp ? f64::ratio_f64_rcp(a, f64::recip_f64((int64_t)b), sh, neg, p, qmin, 127, rf)
                      : f64::ratio_f64(a, b, sh, neg, p, qmin, 127, rf);
    bool bad = false;
    if (c >= 0) {
      const Rnd re = round_ratio64(a, b, sh, neg, p, qmin, 127);
      bad = !rnd_eq(re, rf) || re.ovf;
    }
    tally(acc, c >= 0, bad, (uint64_t)i);
  }
}

}  // namespace
}  // namespace ea

extern "C" int ea_selftest_fast64(int mode, uint64_t seed, uint32_t stride, int64_t n, int64_t* out) {
  if (!out || n < 0 || mode < 0 || mode > 3) return -1;
  unsigned long long* d = nullptr;
  if (cudaMalloc(&d, 4 * sizeof(unsigned long long)) != cudaSuccess) return -4;
  cudaMemset(d, 0, 4 * sizeof(unsigned long long));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (mode == 0)
    ea::selftest_weight_kernel<<<8 * sms, 256>>>((uint32_t)seed, stride ? stride : 1u, n, d);
  else if (mode == 1)
    ea::selftest_logit_kernel<<<8 * sms, 256>>>(seed, n, d);
  else
    ea::selftest_ratio_kernel<<<8 * sms, 256>>>(seed, n, mode == 3, d);
  cudaError_t e = cudaGetLastError();
  unsigned long long h[4] = {0, 0, 0, 0};
  if (e == cudaSuccess) e = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  cudaFree(d);
  for (int i = 0; i < 4; ++i) out[i] = (int64_t)h[i];
  return e == cudaSuccess ? 0 : -4;
}
