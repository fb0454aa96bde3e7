// Deterministic synthetic bf16 tensors for the benchmark and test workloads, bit-identical to the
// numpy generator in exactattention_b200/workloads.py (integer arithmetic only):
//   element i of tensor (seed, id): three splitmix64 hashes -> twelve 16-bit uniforms
//   c = sum - 393210 (Irwin-Hall, approximately N(0, 65536^2))
//   value = RN_bf16(c * mS * 2^(eS - 16)), (mS, eS) the fp32 scale of (head, channel), times 32
//   on the rows a separate hash marks heavy.
// Layout: logical tensor (G, H, T, D) flattened; optionally scattered into paged storage.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/exactattn_synth.h"

namespace {

__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ inline uint16_t rn_bf16(int64_t X, int E) {
  if (X == 0) return 0;
  uint16_t sign = X < 0 ? 0x8000 : 0;
  uint64_t a = X < 0 ? (uint64_t)(-X) : (uint64_t)X;
  int L = 64 - __clzll((long long)a);
  uint64_t q;
  int K = E + L - 1;  // leading exponent
  if (L <= 8) {
    q = a << (8 - L);
  } else {
    int sh = L - 8;
    q = a >> sh;
    uint64_t rem = a & ((1ull << sh) - 1), half = 1ull << (sh - 1);
    if (rem > half || (rem == half && (q & 1))) ++q;
    if (q == 256) {
      q = 128;
      ++K;
    }
  }
  // normal range only (the generators never leave it)
  return (uint16_t)(sign | ((uint16_t)(K + 127) << 7) | (uint16_t)(q & 0x7F));
}

__global__ void synth_kernel(uint16_t* dst, ea_synth_t s) {
  const int64_t total = s.G * s.H * s.T * s.D;
  const uint64_t base = splitmix64(((uint64_t)s.seed << 20) ^ (uint64_t)s.tensor_id);
  const uint64_t hbase = splitmix64(base ^ 0x5555555555555555ull);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t c = i % s.D, t = (i / s.D) % s.T, h = (i / (s.D * s.T)) % s.H, g = i / (s.D * s.T * s.H);
    uint16_t out = 0;
    const int64_t Tf = s.T_full > 0 ? s.T_full : s.T;
    const uint64_t li = (uint64_t)((((g * s.H + h) * Tf) + s.t0 + t) * s.D + c);  // logical index
    if (!s.lens || t < s.lens[g]) {
      uint64_t h0 = splitmix64(base + 3 * li), h1 = splitmix64(base + 3 * li + 1), h2 = splitmix64(base + 3 * li + 2);
      int64_t sum = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        sum += (int64_t)((h0 >> (16 * j)) & 0xFFFF) + (int64_t)((h1 >> (16 * j)) & 0xFFFF) +
               (int64_t)((h2 >> (16 * j)) & 0xFFFF);
      int64_t cv = sum - 393210;
      int64_t sm = s.scale_m ? s.scale_m[h * s.D + c] : (1 << 23);
      int se = s.scale_e ? s.scale_e[h * s.D + c] : -23;
      if (s.heavy_permille > 0 && (splitmix64(hbase + li / (uint64_t)s.D) % 1000) < (uint64_t)s.heavy_permille)
        se += 5;
      out = rn_bf16(cv * sm, se - 16);
    }
    int64_t o = i;
    if (s.page_table) {
      // physical (page, h, slot, c) for logical (g, h, t, c); slots past the sequence stay untouched
      if (t >= s.lens[g]) continue;
      int64_t page = s.page_table[g * s.max_pages + t / s.page_size];
      o = ((page * s.H + h) * s.page_size + (t % s.page_size)) * s.D + c;
    }
    dst[o] = out;
  }
}

}  // namespace

extern "C" int ea_synth_fill(uint16_t* dst, const ea_synth_t* spec, void* stream) {
  if (!dst || !spec || spec->D <= 0) return -1;
  int64_t total = spec->G * spec->H * spec->T * spec->D;
  if (total <= 0) return 0;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 148 * 64) blocks = 148 * 64;
  synth_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(dst, *spec);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
