/* Host form of the synthetic workload generator (benchmarks and tests only): the rows
 * [g, h, t0:t1, :] of the logical (G, H, T, D) tensor, bit-identical to csrc/ea_synth.cu and to
 * the numpy generator in exactattention_b200/workloads.py, on all host threads (OpenMP). The
 * CPU baselines of the long-context configuration need gigabytes of these rows; numpy makes
 * them at about 2 M elements/s. */
#include <stdint.h>

static inline uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* RN-even of X * 2^E to bf16 bits (normal range; the generators never leave it) */
static inline uint16_t rn_bf16(int64_t X, int E) {
  if (X == 0) return 0;
  const uint16_t sign = X < 0 ? 0x8000 : 0;
  const uint64_t a = X < 0 ? (uint64_t)(-X) : (uint64_t)X;
  const int L = 64 - __builtin_clzll(a);
  int K = E + L - 1;
  uint64_t q;
  if (L <= 8) {
    q = a << (8 - L);
  } else {
    const int sh = L - 8;
    q = a >> sh;
    const uint64_t rem = a & ((1ull << sh) - 1), half = 1ull << (sh - 1);
    if (rem > half || (rem == half && (q & 1))) ++q;
    if (q == 256) {
      q = 128;
      ++K;
    }
  }
  return (uint16_t)(sign | ((uint16_t)(K + 127) << 7) | (uint16_t)(q & 0x7F));
}

int ea_synth_rows_host(uint16_t* out, uint64_t seed, uint64_t tensor_id, int64_t H, int64_t T, int64_t D,
                       int64_t g, int64_t h, int64_t t0, int64_t t1, const int32_t* scale_m,
                       const int32_t* scale_e, int heavy_permille) {
  if (!out || D <= 0 || t1 < t0) return -1;
  const uint64_t base = splitmix64((seed << 20) ^ tensor_id);
  const uint64_t hbase = splitmix64(base ^ 0x5555555555555555ull);
  const int64_t n = (t1 - t0) * D;
  const int64_t start = ((g * H + h) * T + t0) * D;
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < n; ++k) {
    const uint64_t li = (uint64_t)(start + k);
    const uint64_t h0 = splitmix64(base + 3 * li), h1 = splitmix64(base + 3 * li + 1),
                   h2 = splitmix64(base + 3 * li + 2);
    int64_t sum = 0;
    for (int j = 0; j < 4; ++j)
      sum += (int64_t)((h0 >> (16 * j)) & 0xFFFF) + (int64_t)((h1 >> (16 * j)) & 0xFFFF) +
             (int64_t)((h2 >> (16 * j)) & 0xFFFF);
    const int64_t c = (int64_t)(li % (uint64_t)D);
    const int64_t sm = scale_m ? scale_m[h * D + c] : (1 << 23);
    int se = scale_e ? scale_e[h * D + c] : -23;
    if (heavy_permille > 0 && (splitmix64(hbase + li / (uint64_t)D) % 1000) < (uint64_t)heavy_permille) se += 5;
    out[k] = rn_bf16((sum - 393210) * sm, se - 16);
  }
  return 0;
}
