// CUDA-core kernels of certified split-KV ExactAttention (tier 1 for any mask, the split combine,
// and the wide-integer tier 3). Tensor-core kernels for the structured masks live in ea_tc.cu.
//
// Tier 1, one warp per (row, KV split), keys in tiles of 32 (one key per lane):
//   score   q and k rows in block fixed point (window W bits below each row's leading bit),
//           acc = sum Qfix Kfix exactly in int64 plus a per-element truncation bound err;
//           t = RN32(alpha s) certified at both ends of [acc - err, acc + err]; otherwise the
//           exact score (576-bit bins) decides (certified.py:93-138 is the reference's model).
//   weight  RN24(2^t) by the 64-bit integer exp2, 128-bit when that is too close to a midpoint.
//   tile    reference exponent Rt = max(E + 24); Z and per-channel N (anchor Rt + VE_c, VE_c the
//           tile's largest |v| exponent in channel c) floor-shifted into int64 windows with
//           lost-bit counts (certified.py:166-210), merged into the running partial
//           (certified.py:213-246).
// Combine: partials of every split are re-expressed at the largest reference exponent and
// summed: integer addition, so the merged state does not depend on split order.
// Finalize: both ends of the N/Z interval rounded; equal ends are the spec's bits
// (certified.py:249-286). Anything uncertified goes to tier 3 on the device.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ea_core.cuh"
#include "ea_numerics.h"
#include "ea_tables.cuh"
#include "ea_wide.h"

namespace ea {

// ---------------------------------------------------------------------------
// shared-memory layout of the tier-1 kernel (host computes the same sizes)
// ---------------------------------------------------------------------------
__host__ __device__ inline int simt_words(int d) { return (d + 1) / 2; }
__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }
__host__ __device__ inline size_t simt_warp_bytes(int d, int dv) {
  size_t qb = align16((size_t)d * 2), qf = align16((size_t)d * 4), ql = align16((size_t)d);
  size_t kt = (size_t)simt_words(d) * 33 * 4, vt = (size_t)32 * dv * 2;
  size_t tile = align16(kt > vt ? kt : vt);
  return qb + qf + ql + tile + 32 * 4 + 32 * 4 + 32 * 4;
}
__host__ __device__ inline size_t simt_smem_bytes(int d, int dv, int warps) {
  return 4096 + (size_t)warps * simt_warp_bytes(d, dv);
}

// warp reductions
__device__ __forceinline__ int64_t warp_sum64(int64_t x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ int warp_max32(int x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x = max(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ int warp_min32(int x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x = min(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Block fixed point of one bf16 value at lsb: sign * trunc(|m| 2^(e - lsb)), and whether bits
// were dropped. Callers guarantee e - lsb <= W - bitlen(|m|) (the value fits the window).
__device__ __forceinline__ int32_t fix_elem(int32_t m, int32_t e, int lsb, int& lost) {
  int32_t mag = m < 0 ? -m : m;
  int sh = e - lsb;
  int32_t f;
  if (sh >= 0) {
    f = mag << sh;
    lost = 0;
  } else {
    int s = -sh;
    f = s >= 31 ? 0 : (mag >> s);
    lost = (s >= 31) ? (mag != 0) : ((f << s) != mag);
  }
  return m < 0 ? -f : f;
}

// merge (Rb, Zb, Zeb) into the running (R, Z, Ze); false on lost headroom
__device__ __forceinline__ bool merge_acc(int32_t& R, int64_t& Z, uint64_t& Ze, int32_t Rb, int64_t Zb, uint64_t Zeb) {
  if (Rb == R_EMPTY) return true;
  if (R == R_EMPTY) {
    R = Rb; Z = Zb; Ze = Zeb;
    return true;
  }
  int32_t Rn = max(R, Rb);
  rescale(Z, Ze, Rn - R);
  rescale(Zb, Zeb, Rn - Rb);
  R = Rn;
  Z += Zb;
  Ze += Zeb;
  return fits63(Z, Ze);
}

// Certified rounding of every channel of a row and the row's flag / tier-3 hand-off.
// NR/N/Ne hold channels lane + 32 i.
template <int CPL>
__device__ void finalize_row(const Prob& P, int64_t r, int status, int32_t R, int64_t Z, uint64_t Ze,
                             const int32_t* NR, const int64_t* N, const uint64_t* Ne, int lane) {
  if (status == ST_DOMAIN) {
    for (int c = lane; c < P.dv; c += 32) write_out(P, r, c, rnd_zero());
    if (lane == 0) {
      P.flags[r] = 2;
      stat_add(P, STAT_DOMAIN_ROWS, 1);
    }
    return;
  }
  bool ok = status == ST_OK;
  Rnd res[CPL];
  if (ok) {
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      res[i] = rnd_zero();
      int c = lane + 32 * i;
      if (c >= P.dv || R == R_EMPTY || NR[i] == R_EMPTY) continue;
      int p = P.fp32 ? FP32_P : BF16_P, qmin = P.fp32 ? FP32_QMIN : BF16_QMIN;
      ok &= certify_ratio(N[i], Ne[i], (int64_t)NR[i] - P.FZ, Z, Ze, (int64_t)R - P.FZ, p, qmin, 127, res[i]);
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  const bool forced = ok && forced_uncertified(P, r);
  if (!ok || forced) {
    if (lane == 0) leave_tier(P, r, forced);
    return;
  }
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    int c = lane + 32 * i;
    if (c < P.dv) write_out(P, r, c, res[i]);
  }
  if (lane == 0) P.flags[r] = 0;
}

// one row's partial into the export buffers (warp per row; NR/N/Ne hold channels lane + 32 i)
template <int CPL>
__device__ void export_row(const Prob& P, int64_t r, int status, int32_t R, int64_t Z, uint64_t Ze,
                           const int32_t* NR, const int64_t* N, const uint64_t* Ne, int lane) {
  if (lane == 0) {
    P.xR[r] = R;
    P.xZ[r] = Z;
    P.xZe[r] = Ze;
    P.xSt[r] = status;
  }
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c >= P.dv) continue;
    P.xNR[r * P.dv + c] = NR[i];
    P.xN[r * P.dv + c] = N[i];
    P.xNe[r * P.dv + c] = Ne[i];
  }
}

// ---------------------------------------------------------------------------
// tier 1 (and tier 2): one warp over a key range of one row
// ---------------------------------------------------------------------------
// The int64 partial of a key range: lane holds channels lane + 32 i.
template <int CPL>
struct SimtPart {
  int status;
  int32_t R, Rlo;  // running reference exponent; lowest E + 24 seen (the logit spread check)
  int64_t Z;
  uint64_t Ze;
  int32_t NR[CPL];
  int64_t N[CPL];
  uint64_t Ne[CPL];
};

// the exp2 tables of the 64-bit weight path into shared memory (4 KB at the start of smem)
__device__ __forceinline__ void load_exp2_tables(uint64_t* sTA, uint64_t* sTB) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    sTA[i] = g_ta64[i];
    sTB[i] = g_tb64[i];
  }
}

// Row r's keys [j0, j1) by one warp on the CUDA cores; ws is the warp's shared workspace
// (simt_warp_bytes). Counts exact scores and wide weights into n_exact / n_wide (this lane).
template <int CPL>
__device__ __forceinline__ void simt_range(const Prob& P, int64_t r, int64_t j0, int64_t j1, const uint64_t* sTA,
                                           const uint64_t* sTB, unsigned char* ws, SimtPart<CPL>& out,
                                           unsigned long long& n_exact, unsigned long long& n_wide) {
  const int lane = threadIdx.x & 31;
  const int d = P.d, dv = P.dv, nw = simt_words(d);
  uint16_t* qbits = (uint16_t*)ws;
  int32_t* qfix = (int32_t*)(ws + align16((size_t)d * 2));
  uint8_t* qlost = (uint8_t*)((unsigned char*)qfix + align16((size_t)d * 4));
  unsigned char* tile = (unsigned char*)qlost + align16((size_t)d);
  size_t kt = (size_t)nw * 33 * 4, vt = (size_t)32 * dv * 2;
  uint32_t* ktile = (uint32_t*)tile;
  uint16_t* vtile = (uint16_t*)tile;
  uint32_t* sM = (uint32_t*)(tile + align16(kt > vt ? kt : vt));
  int32_t* sE = (int32_t*)(sM + 32);

  // ---- q row: decode, leading exponent, block fixed point ----
  int status = ST_OK;
  int qlead = INT32_MIN;
  for (int i = lane; i < d; i += 32) {
    uint16_t b = P.q[r * d + i];
    qbits[i] = b;
    int32_t m, e;
    if (!decode_bf16(b, m, e)) status = ST_DOMAIN;
    if (m) qlead = max(qlead, e + bitlen64((uint64_t)(m < 0 ? -m : m)) - 1);
  }
  qlead = warp_max32(qlead);
  status = warp_max32(status);
  const int qlsb = qlead == INT32_MIN ? 0 : qlead + 1 - P.W;
  for (int i = lane; i < d; i += 32) {
    int32_t m, e;
    decode_bf16(qbits[i], m, e);
    int lost = 0;
    qfix[i] = (m && status == ST_OK) ? fix_elem(m, e, qlsb, lost) : 0;
    qlost[i] = (uint8_t)lost;
  }
  __syncwarp();

  int32_t R = R_EMPTY;
  int32_t Rlo = INT32_MAX;  // lowest E + 24 seen (the logit spread check)
  int64_t Z = 0;
  uint64_t Ze = 0;
  int32_t NR[CPL];
  int64_t N[CPL];
  uint64_t Ne[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    NR[i] = R_EMPTY;
    N[i] = 0;
    Ne[i] = 0;
  }
  const int FZ = P.FZ;

  for (int64_t t0 = j0; t0 < j1 && status == ST_OK; t0 += 32) {
    const int nt = (int)min((int64_t)32, j1 - t0);
    const bool valid = lane < nt;
    const int64_t myrow = valid ? key_row(P, r, t0 + lane) : 0;
    // ---- K tile, transposed into 32-bit words [w][key] (row pitch 33: conflict-free) ----
    for (int jj = 0; jj < nt; ++jj) {
      int64_t kr = __shfl_sync(0xffffffffu, myrow, jj);
      const uint16_t* src = P.k + kr * d;
      for (int w = lane; w < nw; w += 32) {
        uint32_t lo = src[2 * w];
        uint32_t hi = (2 * w + 1 < d) ? src[2 * w + 1] : 0u;
        ktile[w * 33 + jj] = lo | (hi << 16);
      }
    }
    __syncwarp();
    // ---- score, logit, weight of key `lane` ----
    int kst = ST_OK;
    uint32_t M = 0;
    int32_t E = 0;
    if (valid) {
      int klead = INT32_MIN;
      for (int w = 0; w < nw; ++w) {
        uint32_t x = ktile[w * 33 + lane];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int32_t m, e;
          if (!decode_bf16((x >> (16 * h)) & 0xFFFFu, m, e)) kst = ST_DOMAIN;
          if (m) klead = max(klead, e + bitlen64((uint64_t)(m < 0 ? -m : m)) - 1);
        }
      }
      Rnd t = rnd_zero();
      if (kst == ST_OK) {
        const int klsb = klead == INT32_MIN ? 0 : klead + 1 - P.W;
        int64_t acc = 0;
        uint64_t err = 0;
        if (klead != INT32_MIN && qlead != INT32_MIN) {
          for (int w = 0; w < nw; ++w) {
            uint32_t x = ktile[w * 33 + lane];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              int i = 2 * w + h;
              if (i >= d) break;
              int32_t m, e;
              decode_bf16((x >> (16 * h)) & 0xFFFFu, m, e);
              int lost = 0;
              int32_t kf = m ? fix_elem(m, e, klsb, lost) : 0;
              int32_t qf = qfix[i];
              acc += (int64_t)qf * kf;
              err += (uint64_t)qlost[i] * (uint64_t)((kf < 0 ? -kf : kf) + lost) +
                     (uint64_t)lost * (uint64_t)(qf < 0 ? -qf : qf);
            }
          }
        }
        int ls = logit_from_interval(acc, err, qlsb + klsb, P.am, P.ae, t);
        if (ls == LOGIT_UNCERTIFIED) {
          ++n_exact;
          ExactScore sc;
          score_clear(sc);
          for (int i = 0; i < d; ++i) {
            int32_t qm, qe, km, ke;
            decode_bf16(qbits[i], qm, qe);
            decode_bf16((ktile[(i >> 1) * 33 + lane] >> (16 * (i & 1))) & 0xFFFFu, km, ke);
            if (qm && km) score_add(sc, qm * km, qe + ke);
          }
          ls = logit_exact(sc, P.am, P.ae, t);
        }
        if (ls == LOGIT_OVERFLOW) kst = ST_DOMAIN;
      }
      if (kst == ST_OK) {
        int64_t E64;
        int wst = weight_from_logit(t, sTA, sTB, M, E64);
        if (wst == W_RISKY) {
          ++n_wide;
          wst = weight_from_logit_wide(t, g_ta128, g_tb128, M, E64);
        }
        if (wst != W_OK) kst = ST_TIER3;  // |t| >= 2^30 or a still-risky weight
        E = (int32_t)E64;
      }
    }
    kst = warp_max32(kst);
    if (kst != ST_OK) {
      status = kst;
      break;
    }
    // ---- tile partial: Z ----
    int32_t Rt = warp_max32(valid ? E + 24 : INT32_MIN);
    Rlo = min(Rlo, warp_min32(valid ? E + 24 : INT32_MAX));
    int64_t zt = 0;
    int zl = 0;
    if (valid) zt = floor_shift((int64_t)M, E + FZ - Rt, zl);
    int64_t Zt = warp_sum64(zt);
    uint64_t Zet = (uint64_t)warp_sum64(zl);
    if (valid) {
      sM[lane] = M;
      sE[lane] = E;
    }
    __syncwarp();
    // ---- V tile (row-major) over the K tile's space ----
    for (int jj = 0; jj < nt; ++jj) {
      int64_t vr = __shfl_sync(0xffffffffu, myrow, jj);
      const uint16_t* src = P.v + vr * dv;
      for (int c = lane; c < dv; c += 32) vtile[jj * dv + c] = src[c];
    }
    __syncwarp();
    bool ok = merge_acc(R, Z, Ze, Rt, Zt, Zet);
    int vst = ST_OK;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      int c = lane + 32 * i;
      if (c >= dv) continue;
      int VE = INT32_MIN;
      for (int jj = 0; jj < nt; ++jj) {
        int32_t m, e;
        if (!decode_bf16(vtile[jj * dv + c], m, e)) vst = ST_DOMAIN;
        if (m) VE = max(VE, e + bitlen64((uint64_t)(m < 0 ? -m : m)));
      }
      if (VE == INT32_MIN) continue;
      int32_t NRt = Rt + VE;
      int64_t acc = 0;
      uint64_t err = 0;
      for (int jj = 0; jj < nt; ++jj) {
        int32_t m, e;
        decode_bf16(vtile[jj * dv + c], m, e);
        if (!m) continue;
        int lost;
        acc += floor_shift((int64_t)sM[jj] * m, sE[jj] + e - NRt + FZ, lost);
        err += (uint64_t)lost;
      }
      ok &= merge_acc(NR[i], N[i], Ne[i], NRt, acc, err);
    }
    vst = warp_max32(vst);
    if (vst != ST_OK) status = vst;
    if (!__all_sync(0xffffffffu, ok) && status == ST_OK) status = ST_TIER3;
    __syncwarp();
  }
  status = warp_max32(status);
  if (status == ST_OK && R != R_EMPTY && Rlo != INT32_MAX && (int64_t)R - Rlo > SPREAD_CHECK) status = ST_TIER3;
  out.status = status;
  out.R = R;
  out.Rlo = Rlo;
  out.Z = Z;
  out.Ze = Ze;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    out.NR[i] = NR[i];
    out.N[i] = N[i];
    out.Ne[i] = Ne[i];
  }
}

// the counters of one warp's range (lane 0 adds the warp's sums)
__device__ __forceinline__ void simt_stats(const Prob& P, unsigned long long n_exact, unsigned long long n_wide,
                                           unsigned long long pairs, int pairs_slot) {
  n_exact = (unsigned long long)warp_sum64((int64_t)n_exact);
  n_wide = (unsigned long long)warp_sum64((int64_t)n_wide);
  if ((threadIdx.x & 31) == 0) {
    stat_add(P, STAT_SCORE_EXACT, n_exact);
    stat_add(P, STAT_WEIGHT_WIDE, n_wide);
    stat_add(P, pairs_slot, pairs);
  }
}

// one partial into slot pi of the split (or unit) buffers P.p*
template <int CPL>
__device__ __forceinline__ void write_split_partial(const Prob& P, int64_t pi, const SimtPart<CPL>& o) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) {
    P.pR[pi] = o.R;
    P.pZ[pi] = o.Z;
    P.pZe[pi] = o.Ze;
    P.pSt[pi] = o.status;
  }
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c >= P.dv) continue;
    P.pNR[pi * P.dv + c] = o.NR[i];
    P.pN[pi * P.dv + c] = o.N[i];
    P.pNe[pi * P.dv + c] = o.Ne[i];
  }
}

// ---------------------------------------------------------------------------
// tier 1: one warp per (row, KV split)
// ---------------------------------------------------------------------------
template <int CPL>
__global__ void __launch_bounds__(128) simt_split_kernel(Prob P) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  uint64_t* sTA = (uint64_t*)smem;
  uint64_t* sTB = sTA + 256;
  load_exp2_tables(sTA, sTB);
  __syncthreads();
  unsigned char* ws = smem + 4096 + (size_t)warp * simt_warp_bytes(P.d, P.dv);
  const int64_t r = (int64_t)blockIdx.x * nwarps + warp;
  if (r >= P.rows) return;
  const int S = P.splits, s = blockIdx.y;
  const int64_t L = row_len(P, r);
  const int64_t j0 = L * s / S, j1 = L * (s + 1) / S;
  SimtPart<CPL> o;
  unsigned long long n_exact = 0, n_wide = 0;
  simt_range<CPL>(P, r, j0, j1, sTA, sTB, ws, o, n_exact, n_wide);
  simt_stats(P, n_exact, n_wide, (unsigned long long)(j1 - j0), STAT_PAIRS);
  const int status = o.status;
  const int32_t R = o.R;
  const int64_t Z = o.Z;
  const uint64_t Ze = o.Ze;
  const int32_t* NR = o.NR;
  const int64_t* N = o.N;
  const uint64_t* Ne = o.Ne;
  if (S == 1) {
    if (P.export_partials)
      export_row<CPL>(P, r, status, R, Z, Ze, NR, N, Ne, lane);
    else
      finalize_row<CPL>(P, r, status, R, Z, Ze, NR, N, Ne, lane);
    return;
  }
  write_split_partial<CPL>(P, (int64_t)s * P.rows + r, o);
  (void)lane;
}

// ---------------------------------------------------------------------------
// split combine: max reference exponent, rescale, integer sum (order-independent)
// ---------------------------------------------------------------------------
// Merge of the partials in slots first + s * stride (s < S), one warp: the largest reference
// exponents, every partial re-expressed at them, integer sums (order-free), the spread check.
// pRlo (optional): per slot the lowest reference exponent among the partials merged into it
// before (a two-level merge), so that the spread check sees every original partial.
template <int CPL>
__device__ __forceinline__ void merge_slots(const Prob& P, int64_t first, int64_t stride, int S, SimtPart<CPL>& o,
                                            const int32_t* pRlo = nullptr) {
  const int lane = threadIdx.x & 31;
  const int dv = P.dv;
  int status = ST_OK;
  int32_t R = R_EMPTY, Rmin = INT32_MAX;
  for (int s = 0; s < S; ++s) {
    int64_t pi = first + (int64_t)s * stride;
    status = max(status, P.pSt[pi]);
    if (P.pR[pi] != R_EMPTY) {
      R = (R == R_EMPTY) ? P.pR[pi] : max(R, P.pR[pi]);
      Rmin = min(Rmin, pRlo ? pRlo[pi] : P.pR[pi]);
    }
  }
  // a split far below the row's largest weights: the exponent spread may exceed the reference's
  // limit (tier 3 decides)
  if (status == ST_OK && R != R_EMPTY && (int64_t)R - Rmin > SPREAD_CHECK) status = ST_TIER3;
  int64_t Z = 0;
  uint64_t Ze = 0;
  bool ok = true;
  if (status == ST_OK && R != R_EMPTY) {
    for (int s = 0; s < S; ++s) {
      int64_t pi = first + (int64_t)s * stride;
      if (P.pR[pi] == R_EMPTY) continue;
      int64_t z = P.pZ[pi];
      uint64_t ze = P.pZe[pi];
      rescale(z, ze, R - P.pR[pi]);
      Z += z;
      Ze += ze;
    }
    ok &= fits63(Z, Ze);
  }
  int32_t NR[CPL];
  int64_t N[CPL];
  uint64_t Ne[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    NR[i] = R_EMPTY;
    N[i] = 0;
    Ne[i] = 0;
    int c = lane + 32 * i;
    if (c >= dv || status != ST_OK) continue;
    for (int s = 0; s < S; ++s) {
      int32_t x = P.pNR[(first + (int64_t)s * stride) * dv + c];
      if (x != R_EMPTY) NR[i] = NR[i] == R_EMPTY ? x : max(NR[i], x);
    }
    if (NR[i] == R_EMPTY) continue;
    for (int s = 0; s < S; ++s) {
      int64_t pc = (first + (int64_t)s * stride) * dv + c;
      int32_t x = P.pNR[pc];
      if (x == R_EMPTY) continue;
      int64_t n = P.pN[pc];
      uint64_t ne = P.pNe[pc];
      rescale(n, ne, NR[i] - x);
      N[i] += n;
      Ne[i] += ne;
    }
    ok &= fits63(N[i], Ne[i]);
  }
  if (!__all_sync(0xffffffffu, ok) && status == ST_OK) status = ST_TIER3;
  o.status = status;
  o.R = R;
  o.Rlo = Rmin;
  o.Z = Z;
  o.Ze = Ze;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    o.NR[i] = NR[i];
    o.N[i] = N[i];
    o.Ne[i] = Ne[i];
  }
}

template <int CPL>
__global__ void __launch_bounds__(128) combine_kernel(Prob P) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (r >= P.rows) return;
  SimtPart<CPL> o;
  merge_slots<CPL>(P, r, P.rows, P.splits, o);
  if (P.export_partials)
    export_row<CPL>(P, r, o.status, o.R, o.Z, o.Ze, o.NR, o.N, o.Ne, lane);
  else
    finalize_row<CPL>(P, r, o.status, o.R, o.Z, o.Ze, o.NR, o.N, o.Ne, lane);
}

// The same split combine with a block of 128 threads per row (dv <= 128): warp 0 merges the row's
// exponents, status and Z over the splits (lane-strided, then warp reductions: integer sums taken
// modulo 2^64 are order-free, so the bits equal the sequential merge's), thread c merges channel c,
// and the fits / certification votes cover the whole block. Rows with few splits' worth of work
// each (a long decode row cut into 32 splits) no longer wait on one warp's serial loop over
// splits x channels.
__global__ void __launch_bounds__(128) combine_row_kernel(Prob P) {
  __shared__ int32_t s_R, s_st;
  __shared__ int64_t s_Z;
  __shared__ uint64_t s_Ze;
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t r = blockIdx.x;
  const int S = P.splits, dv = P.dv;
  const int64_t stride = P.rows;
  if (tid < 32) {
    int status = ST_OK;
    int32_t R = R_EMPTY, Rmin = INT32_MAX;  // R_EMPTY is INT32_MIN: below every exponent
    for (int s = lane; s < S; s += 32) {
      const int64_t pi = r + (int64_t)s * stride;
      status = max(status, P.pSt[pi]);
      const int32_t x = P.pR[pi];
      if (x != R_EMPTY) {
        R = max(R, x);
        Rmin = min(Rmin, x);
      }
    }
    status = __reduce_max_sync(0xffffffffu, status);
    R = __reduce_max_sync(0xffffffffu, R);
    Rmin = __reduce_min_sync(0xffffffffu, Rmin);
    if (status == ST_OK && R != R_EMPTY && (int64_t)R - Rmin > SPREAD_CHECK) status = ST_TIER3;
    int64_t Z = 0;
    uint64_t Ze = 0;
    if (status == ST_OK && R != R_EMPTY) {
      for (int s = lane; s < S; s += 32) {
        const int64_t pi = r + (int64_t)s * stride;
        if (P.pR[pi] == R_EMPTY) continue;
        int64_t z = P.pZ[pi];
        uint64_t ze = P.pZe[pi];
        rescale(z, ze, R - P.pR[pi]);
        Z += z;
        Ze += ze;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        Z += __shfl_xor_sync(0xffffffffu, Z, o);
        Ze += __shfl_xor_sync(0xffffffffu, Ze, o);
      }
    }
    if (lane == 0) {
      s_R = R;
      s_st = status;
      s_Z = Z;
      s_Ze = Ze;
    }
  }
  __syncthreads();
  const int32_t R = s_R;
  const int64_t Z = s_Z;
  const uint64_t Ze = s_Ze;
  int status = s_st;
  bool ok = true;
  if (status == ST_OK && R != R_EMPTY) ok = fits63(Z, Ze);
  const int c = tid;
  int32_t NR = R_EMPTY;
  int64_t N = 0;
  uint64_t Ne = 0;
  if (c < dv && status == ST_OK) {
    for (int s = 0; s < S; ++s) {
      const int32_t x = P.pNR[(r + (int64_t)s * stride) * dv + c];
      if (x != R_EMPTY) NR = max(NR, x);
    }
    if (NR != R_EMPTY) {
      for (int s = 0; s < S; ++s) {
        const int64_t pc = (r + (int64_t)s * stride) * dv + c;
        const int32_t x = P.pNR[pc];
        if (x == R_EMPTY) continue;
        int64_t n = P.pN[pc];
        uint64_t ne = P.pNe[pc];
        rescale(n, ne, NR - x);
        N += n;
        Ne += ne;
      }
      ok &= fits63(N, Ne);
    }
  }
  if (!__syncthreads_and(ok) && status == ST_OK) status = ST_TIER3;
  if (P.export_partials) {
    if (tid == 0) {
      P.xR[r] = R;
      P.xZ[r] = Z;
      P.xZe[r] = Ze;
      P.xSt[r] = status;
    }
    if (c < dv) {
      P.xNR[r * dv + c] = NR;
      P.xN[r * dv + c] = N;
      P.xNe[r * dv + c] = Ne;
    }
    return;
  }
  if (status == ST_DOMAIN) {
    if (c < dv) write_out(P, r, c, rnd_zero());
    if (tid == 0) {
      P.flags[r] = 2;
      stat_add(P, STAT_DOMAIN_ROWS, 1);
    }
    return;
  }
  bool cert = status == ST_OK;
  Rnd res = rnd_zero();
  if (cert && c < dv && R != R_EMPTY && NR != R_EMPTY) {
    const int p = P.fp32 ? FP32_P : BF16_P, qmin = P.fp32 ? FP32_QMIN : BF16_QMIN;
    cert = certify_ratio(N, Ne, (int64_t)NR - P.FZ, Z, Ze, (int64_t)R - P.FZ, p, qmin, 127, res);
  }
  cert = __syncthreads_and(cert);
  const bool forced = cert && forced_uncertified(P, r);
  if (!cert || forced) {
    if (tid == 0) leave_tier(P, r, forced);
    return;
  }
  if (c < dv) write_out(P, r, c, res);
  if (tid == 0) P.flags[r] = 0;
}

// ---------------------------------------------------------------------------
// tier 2: the rows tier 1 left uncertified, int64 fixed point on the CUDA cores, each row's keys
// cut into chunks over the whole GPU (the reference reruns its uncertified pairs with int64 P.V
// from a device work list: triton_kernels.py:1046-1067, 1498-1515)
// ---------------------------------------------------------------------------
// Plan of a split-K fallback tier, one block of 1024 threads, from device-side counts only (no host
// synchronisation): the rows in_list[0 .. n) with n = min(*in_count, max_rows) get units of
// `chunk` keys, chunk >= min_chunk chosen so that every unit fits ucap; u_off[i] is row i's first
// unit, u_off[n] the unit count; u_n = {n, units, chunk, mode}. Rows past max_rows: mode 0 (tier
// 2) appends them to (over_list, over_count) for tier 3; mode 1 (tier 3) plans no units and marks
// the run as one block per whole row (u_n = {count, count, 0, 1}).
__global__ void __launch_bounds__(1024) fallback_plan_kernel(Prob P, const int* in_list, const int* in_count,
                                                              int max_rows, int ucap, int64_t min_chunk, int* u_off,
                                                              int64_t* u_n, int* over_list, int* over_count,
                                                              int mode) {
  __shared__ int64_t wsum[32];
  __shared__ int64_t s_chunk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int count = *in_count;
  if (mode == 1 && count > max_rows) {
    if (tid == 0) {
      u_n[0] = count;
      u_n[1] = count;
      u_n[2] = 0;
      u_n[3] = 1;
    }
    return;
  }
  const int n = min(count, max_rows);
  for (int i = n + tid; i < count; i += blockDim.x) {
    const int k = atomicAdd(over_count, 1);
    over_list[k] = in_list[i];
  }
  if (tid == 0 && count > n) stat_add(P, STAT_TIER2_UNCERT, (unsigned long long)(count - n));
  // total keys of the planned rows
  int64_t t = 0;
  for (int i = tid; i < n; i += blockDim.x) t += row_len(P, in_list[i]);
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (lane == 0) wsum[warp] = t;
  __syncthreads();
  if (tid == 0) {
    int64_t tot = 0;
    for (int w = 0; w < 32; ++w) tot += wsum[w];
    const int64_t room = max(1, ucap - n);
    s_chunk = max(min_chunk, (tot + room - 1) / room);
  }
  __syncthreads();
  const int64_t chunk = s_chunk;
  // units per row, exclusive scan over contiguous per-thread ranges (sum <= ucap: ceil(L / chunk)
  // <= L / chunk + 1 and the keys fill at most ucap - n chunks)
  const int per = (n + 1023) / 1024;
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  int64_t mine = 0;
  for (int i = i0; i < i1; ++i) {
    const int64_t L = row_len(P, in_list[i]);
    mine += L > chunk ? (L + chunk - 1) / chunk : 1;
  }
  int64_t inc = mine;
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  __syncthreads();
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  int64_t base = inc - mine;
  for (int w = 0; w < warp; ++w) base += wsum[w];
  for (int i = i0; i < i1; ++i) {
    u_off[i] = (int)base;
    const int64_t L = row_len(P, in_list[i]);
    base += L > chunk ? (L + chunk - 1) / chunk : 1;
  }
  if (tid == 1023) {
    u_off[n] = (int)base;  // the last thread's running sum is the total
    u_n[0] = n;
    u_n[1] = base;
    u_n[2] = chunk;
    u_n[3] = 0;
  }
}

// the listed row (index into u_rows) that unit u belongs to: the last i with u_off[i] <= u
__device__ __forceinline__ int unit_row(const int* u_off, int n, int64_t u) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (u_off[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Tier-2 units: warp per (row, key chunk), the tier-1 CUDA-core arithmetic over the chunk; the
// partial goes to the unit's slot of P.p* (grid-stride over the planned units).
template <int CPL>
__global__ void __launch_bounds__(128) tier2_units_kernel(Prob P) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  uint64_t* sTA = (uint64_t*)smem;
  uint64_t* sTB = sTA + 256;
  load_exp2_tables(sTA, sTB);
  __syncthreads();
  unsigned char* ws = smem + 4096 + (size_t)warp * simt_warp_bytes(P.d, P.dv);
  const int n = (int)P.u_n[0];
  const int64_t units = P.u_n[1], chunk = P.u_n[2];
  for (int64_t u = (int64_t)blockIdx.x * nwarps + warp; u < units; u += (int64_t)gridDim.x * nwarps) {
    const int i = unit_row(P.u_off, n, u);
    const int64_t r = P.u_rows[i];
    const int64_t L = row_len(P, r);
    const int64_t j0 = min(L, (u - P.u_off[i]) * chunk), j1 = min(L, j0 + chunk);
    SimtPart<CPL> o;
    unsigned long long n_exact = 0, n_wide = 0;
    simt_range<CPL>(P, r, j0, j1, sTA, sTB, ws, o, n_exact, n_wide);
    simt_stats(P, n_exact, n_wide, (unsigned long long)(j1 - j0), STAT_TIER2_PAIRS);
    write_split_partial<CPL>(P, u, o);
    __syncwarp();
  }
}

// The merge of a row's units runs in two levels so that a long row's thousands of units are
// merged in parallel: groups of GROUP consecutive units are merged in place into their first
// unit's slot (warp per group), then each row merges its group heads. Re-expressing at a group's
// largest exponent and then at the row's is the same floor as one shift (only the error bounds,
// which can only decide whether a row certifies, gain their rounding units).
constexpr int T2_GROUP = 64, T3_GROUP = 16;

// Level 1 of the tier-2 merge: warp per group head (unit u with (u - u_off[i]) % T2_GROUP == 0).
// pRlo[u] keeps the group's lowest exponent for the spread check.
template <int CPL>
__global__ void __launch_bounds__(128) tier2_group_kernel(Prob P, int32_t* pRlo) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int n = (int)P.u_n[0];
  const int64_t units = P.u_n[1];
  for (int64_t u = (int64_t)blockIdx.x * nwarps + warp; u < units; u += (int64_t)gridDim.x * nwarps) {
    const int i = unit_row(P.u_off, n, u);
    if ((u - P.u_off[i]) % T2_GROUP != 0) continue;  // uniform across the warp
    const int cnt = (int)min((int64_t)T2_GROUP, (int64_t)P.u_off[i + 1] - u);
    SimtPart<CPL> o;
    merge_slots<CPL>(P, u, 1, cnt, o);
    __syncwarp();  // every lane has read the group's slots before the head is overwritten
    write_split_partial<CPL>(P, u, o);
    if (lane == 0) pRlo[u] = o.Rlo;
  }
}

// Tier-2 merge, level 2: warp per planned row, its group heads merged exactly and the row
// certified; what still fails goes on to tier 3's list (P.t3_list; P.tier == 2).
template <int CPL>
__global__ void __launch_bounds__(128) tier2_merge_kernel(Prob P, const int32_t* pRlo) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n = P.u_n[0];
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; i < n; i += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t r = P.u_rows[i];
    const int u0 = P.u_off[i], u1 = P.u_off[i + 1];
    SimtPart<CPL> o;
    merge_slots<CPL>(P, u0, T2_GROUP, (u1 - u0 + T2_GROUP - 1) / T2_GROUP, o, pRlo);
    finalize_row<CPL>(P, r, o.status, o.R, o.Z, o.Ze, o.NR, o.N, o.Ne, lane);
  }
}

// ---------------------------------------------------------------------------
// partials of KV shards: re-express at the global exponents, then finalise after the sum
// ---------------------------------------------------------------------------
// Thread per (row, channel); channel 0's thread also handles Z. Exponents Rg/NRg come from an
// all-reduce MAX over the shards; an empty partial (R_EMPTY) contributes zeros. After this every
// shard's integers are in the same units, so their sum (an all-reduce SUM) is order-free.
__global__ void partials_rescale_kernel(Prob P, const int32_t* Rg, const int32_t* NRg) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P.rows * P.dv) return;
  const int64_t r = i / P.dv;
  const int c = (int)(i - r * P.dv);
  if (c == 0) {
    const int32_t R = P.xR[r], G = Rg[r];
    if (R == R_EMPTY) {
      P.xZ[r] = 0;
      P.xZe[r] = 0;
    } else if (G != R_EMPTY && G > R) {
      int64_t z = P.xZ[r];
      uint64_t ze = P.xZe[r];
      rescale(z, ze, G - R);
      if ((int64_t)G - R > SPREAD_CHECK) ze += SPREAD_MARK;  // far below the row's maximum: mark
      P.xZ[r] = z;
      P.xZe[r] = ze;
    }
    P.xR[r] = G;
  }
  const int32_t NR = P.xNR[i], G = NRg[i];
  if (NR == R_EMPTY) {
    P.xN[i] = 0;
    P.xNe[i] = 0;
  } else if (G != R_EMPTY && G > NR) {
    int64_t n = P.xN[i];
    uint64_t ne = P.xNe[i];
    rescale(n, ne, G - NR);
    P.xN[i] = n;
    P.xNe[i] = ne;
  }
  P.xNR[i] = G;
}

// Certified rounding of summed partials (warp per row). A row no tier-1 bound certifies is
// flagged 1 (and counted as a tier-3 row): the sharded wide tier finishes it.
template <int CPL>
__global__ void __launch_bounds__(128) partials_finalize_kernel(Prob P) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (r >= P.rows) return;
  const int status = P.xSt[r];
  const int32_t R = P.xR[r];
  const int64_t Z = P.xZ[r];
  const uint64_t Ze = P.xZe[r];
  if (status == ST_DOMAIN) {
    for (int c = lane; c < P.dv; c += 32) write_out(P, r, c, rnd_zero());
    if (lane == 0) P.flags[r] = 2;
    return;
  }
  // (a shard marked its partial far below the row's maximum: the wide tier decides the spread)
  bool ok = status == ST_OK && (R == R_EMPTY || (fits63(Z, Ze) && Ze < SPREAD_MARK));
  Rnd res[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    res[i] = rnd_zero();
    const int c = lane + 32 * i;
    if (c >= P.dv || !ok || R == R_EMPTY) continue;
    const int32_t NR = P.xNR[r * P.dv + c];
    if (NR == R_EMPTY) continue;
    const int64_t N = P.xN[r * P.dv + c];
    const uint64_t Ne = P.xNe[r * P.dv + c];
    const int p = P.fp32 ? FP32_P : BF16_P, qmin = P.fp32 ? FP32_QMIN : BF16_QMIN;
    ok &= fits63(N, Ne) && certify_ratio(N, Ne, (int64_t)NR - P.FZ, Z, Ze, (int64_t)R - P.FZ, p, qmin, 127, res[i]);
  }
  ok = __all_sync(0xffffffffu, ok);
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c < P.dv) write_out(P, r, c, ok ? res[i] : rnd_zero());
  }
  if (lane == 0) {
    P.flags[r] = ok ? 0 : 1;
    if (!ok) stat_add(P, STAT_TIER3_ROWS, 1);
  }
}

// ---------------------------------------------------------------------------
// the one-collective KV-shard merge: every rank's partials gathered back to back, merged and
// rounded in one kernel (warp per row)
// ---------------------------------------------------------------------------
// Flat layout of one rank's partials (rows, dv): int64 Z[rows], Zerr[rows], N[rows dv],
// Nerr[rows dv], then int32 R[rows], status[rows], NR[rows dv]; stride: the padded rank size.
template <int CPL>
__global__ void __launch_bounds__(128) gathered_merge_kernel(Prob P, const unsigned char* g, int world,
                                                              int64_t stride, int* wide_rows, int* wide_count) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (r >= P.rows) return;
  const int64_t rows = P.rows;
  const int dv = P.dv;
  const int64_t oZe = 8 * rows, oN = 16 * rows, oNe = oN + 8 * rows * dv, oR = oNe + 8 * rows * dv;
  const int64_t oSt = oR + 4 * rows, oNR = oSt + 4 * rows;
  auto i64 = [&](int s, int64_t off, int64_t i) { return ((const int64_t*)(g + s * stride + off))[i]; };
  auto i32 = [&](int s, int64_t off, int64_t i) { return ((const int32_t*)(g + s * stride + off))[i]; };
  int status = ST_OK;
  int32_t R = R_EMPTY, Rmin = INT32_MAX;
  for (int s = 0; s < world; ++s) {
    status = max(status, i32(s, oSt, r));
    const int32_t Rs = i32(s, oR, r);
    if (Rs != R_EMPTY) {
      R = R == R_EMPTY ? Rs : max(R, Rs);
      Rmin = min(Rmin, Rs);
    }
  }
  // a shard far below the row's largest weights: the wide tier decides the exponent spread
  if (status == ST_OK && R != R_EMPTY && (int64_t)R - Rmin > SPREAD_CHECK) status = ST_TIER3;
  int64_t Z = 0;
  uint64_t Ze = 0;
  bool ok = true;
  if (status == ST_OK && R != R_EMPTY) {
    for (int s = 0; s < world; ++s) {
      const int32_t Rs = i32(s, oR, r);
      if (Rs == R_EMPTY) continue;
      int64_t z = i64(s, 0, r);
      uint64_t ze = (uint64_t)i64(s, oZe, r);
      rescale(z, ze, R - Rs);
      Z += z;
      Ze += ze;
    }
    ok &= fits63(Z, Ze);
  }
  Rnd res[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    res[i] = rnd_zero();
    const int c = lane + 32 * i;
    if (c >= dv || status != ST_OK || R == R_EMPTY) continue;
    int32_t NR = R_EMPTY;
    for (int s = 0; s < world; ++s) {
      const int32_t x = i32(s, oNR, r * dv + c);
      if (x != R_EMPTY) NR = NR == R_EMPTY ? x : max(NR, x);
    }
    if (NR == R_EMPTY) continue;
    int64_t N = 0;
    uint64_t Ne = 0;
    for (int s = 0; s < world; ++s) {
      const int32_t x = i32(s, oNR, r * dv + c);
      if (x == R_EMPTY) continue;
      int64_t n = i64(s, oN, r * dv + c);
      uint64_t ne = (uint64_t)i64(s, oNe, r * dv + c);
      rescale(n, ne, NR - x);
      N += n;
      Ne += ne;
    }
    const int p = P.fp32 ? FP32_P : BF16_P, qmin = P.fp32 ? FP32_QMIN : BF16_QMIN;
    ok &= fits63(N, Ne) && certify_ratio(N, Ne, (int64_t)NR - P.FZ, Z, Ze, (int64_t)R - P.FZ, p, qmin, 127, res[i]);
  }
  if (status == ST_DOMAIN) {
    for (int c = lane; c < dv; c += 32) write_out(P, r, c, rnd_zero());
    if (lane == 0) {
      P.flags[r] = 2;
      stat_add(P, STAT_DOMAIN_ROWS, 1);
    }
    return;
  }
  ok = __all_sync(0xffffffffu, ok && status == ST_OK);
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c < dv) write_out(P, r, c, ok ? res[i] : rnd_zero());
  }
  if (lane == 0) {
    P.flags[r] = ok ? 0 : 1;
    if (!ok) stat_add(P, STAT_TIER1_UNCERT, 1);
  }
}

// The rows flagged 1, in increasing row order (every rank must list the wide tier's rows in the
// same order: its SUM all-reduce adds the ranks' partials slot by slot), then -1 in every unused
// slot up to `rows`. One block; a block-wide prefix count per chunk of rows.
__global__ void __launch_bounds__(1024) list_flagged_kernel(const uint8_t* flags, int64_t rows, int* list, int* count) {
  __shared__ int wsum[32];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int64_t r0 = 0; r0 < rows; r0 += 1024) {
    const int64_t r = r0 + tid;
    const bool f = r < rows && flags[r] == 1;
    const unsigned b = __ballot_sync(0xffffffffu, f);
    if (lane == 0) wsum[warp] = __popc(b);
    __syncthreads();
    int before = s_base;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    if (f) list[before + __popc(b & ((1u << lane) - 1))] = (int)r;
    __syncthreads();
    if (tid == 0) {
      int t = 0;
      for (int w = 0; w < 32; ++w) t += wsum[w];
      s_base += t;
    }
    __syncthreads();
  }
  const int n = s_base;
  for (int64_t i = n + tid; i < rows; i += 1024) list[i] = -1;
  if (tid == 0) *count = n;
}

cudaError_t launch_gathered_merge(const Prob& P, const void* g, int world, int64_t stride, int* wide_rows,
                                  int* wide_count, cudaStream_t st) {
  const unsigned gr = (unsigned)((P.rows + 3) / 4);
  const unsigned char* gb = (const unsigned char*)g;
  if (P.dv <= 32) gathered_merge_kernel<1><<<gr, 128, 0, st>>>(P, gb, world, stride, wide_rows, wide_count);
  else if (P.dv <= 64) gathered_merge_kernel<2><<<gr, 128, 0, st>>>(P, gb, world, stride, wide_rows, wide_count);
  else if (P.dv <= 128) gathered_merge_kernel<4><<<gr, 128, 0, st>>>(P, gb, world, stride, wide_rows, wide_count);
  else gathered_merge_kernel<8><<<gr, 128, 0, st>>>(P, gb, world, stride, wide_rows, wide_count);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  list_flagged_kernel<<<1, 1024, 0, st>>>(P.flags, P.rows, wide_rows, wide_count);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// tier 3: one block per listed row, wide fixed point over every key of the row
// ---------------------------------------------------------------------------
// Weights: the same certified logit (exact score when the window does not decide) and the
// 128-bit exp2. Exponents are int64, so |t| up to 2^62 is handled; beyond that, or past the
// reference's exponent-spread limit (reference.py:30, 116-118), the row is a domain error.
// Accumulators: Z and each channel's N in Wide<LW> windows, Z in units 2^(R - FW) and N in units
// 2^(R + 128 - FW) (|v| < 2^128), R the running reference exponent. Terms within about
// 32 LW - 64 - key_log2 - 160 bits of the largest are kept exactly.
constexpr int T3_THREADS = 128;
constexpr int LW = 48;                 // 1536-bit windows
constexpr int64_t MAX_SPREAD = 1ll << 20;

__device__ __forceinline__ int64_t block_max64(int64_t x, int64_t* red) {
  for (int o = 16; o; o >>= 1) x = max(x, (int64_t)__shfl_xor_sync(0xffffffffu, x, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  int64_t m = red[0];
  for (int i = 1; i < T3_THREADS / 32; ++i) m = max(m, red[i]);
  __syncthreads();
  return m;
}

// RN of N / Z from the wide intervals N in [N, N + Nerr] (units 2^(R + 128 - FW)) and Z in
// [Z, Z + Zerr] (units 2^(R - FW)), both normalised: true (and res) when both ends round alike.
__device__ bool wide_round(const Prob& P, const Wide<LW>& Zw, uint64_t Zerr, const Wide<LW>& Nw, uint64_t Nerr,
                           Rnd& res) {
  uint32_t za[LW + 1], zb[LW + 1], na[LW + 1];
  Zw.magnitude(za);
  for (int i = 0; i <= LW; ++i) zb[i] = za[i];
  big_add_u64(zb, LW + 1, Zerr);
  bool nneg = Nw.magnitude(na);
  uint32_t nlo[LW + 1], nhi[LW + 1];
  const int p = P.fp32 ? FP32_P : BF16_P, qmin = P.fp32 ? FP32_QMIN : BF16_QMIN;
  Rnd rl, rh;
  if (!nneg) {
    for (int i = 0; i <= LW; ++i) nlo[i] = nhi[i] = na[i];
    big_add_u64(nhi, LW + 1, Nerr);
    rl = round_ratio_big<LW + 4>(nlo, zb, LW + 1, 128, 0, p, qmin, 127);
    rh = round_ratio_big<LW + 4>(nhi, za, LW + 1, 128, 0, p, qmin, 127);
  } else {
    // N = -|N|; the high end N + Nerr may cross zero
    for (int i = 0; i <= LW; ++i) nlo[i] = na[i];
    rl = round_ratio_big<LW + 4>(nlo, za, LW + 1, 128, 1, p, qmin, 127);
    // |N| - Nerr, or Nerr - |N| if that is negative
    uint32_t e[LW + 1];
    for (int i = 0; i <= LW; ++i) e[i] = 0;
    big_add_u64(e, LW + 1, Nerr);
    if (big_cmp(na, e, LW + 1) >= 0) {
      for (int i = 0; i <= LW; ++i) nhi[i] = na[i];
      big_sub(nhi, e, LW + 1);
      rh = round_ratio_big<LW + 4>(nhi, zb, LW + 1, 128, 1, p, qmin, 127);
    } else {
      for (int i = 0; i <= LW; ++i) nhi[i] = e[i];
      big_sub(nhi, na, LW + 1);
      rh = round_ratio_big<LW + 4>(nhi, za, LW + 1, 128, 0, p, qmin, 127);
    }
  }
  res = rl;
  if (res.q == 0) res.neg = 0;
  return rnd_eq(rl, rh);
}

__global__ void __launch_bounds__(T3_THREADS) tier3_kernel(Prob P) {
  __shared__ uint32_t sM[T3_THREADS];
  __shared__ int64_t sE[T3_THREADS];
  __shared__ int64_t sRow[T3_THREADS];
  __shared__ int64_t red[T3_THREADS / 32];
  __shared__ int sStatus;
  const int tid = threadIdx.x;
  const int d = P.d, dv = P.dv;
  const int64_t FW = 32ll * LW - 64 - P.key_log2;
  // planned run (after tier 2): u_n[3] == 0 split-K units (item = unit, its key chunk, a wide
  // partial per unit for tier3_merge_kernel), 1 one item per listed row; otherwise the list
  // (t3_list, t3_count or t3_fixed) with whole rows
  const bool planned = P.u_n != nullptr;
  const bool split = planned && P.u_n[3] == 0;
  const bool exporting = P.export_partials || split;
  const int count = planned ? (int)P.u_n[1] : P.t3_fixed > 0 ? P.t3_fixed : *P.t3_count;

  for (int item = blockIdx.x; item < count; item += gridDim.x) {
    int64_t r, j0 = 0, j1;
    if (split) {
      const int i = unit_row(P.u_off, (int)P.u_n[0], item);
      r = P.u_rows[i];
      const int64_t L = row_len(P, r);
      j0 = min(L, (item - P.u_off[i]) * P.u_n[2]);
      j1 = min(L, j0 + P.u_n[2]);
    } else {
      r = planned ? P.u_rows[item] : P.t3_list[item];
      if (r < 0) {  // an unused slot of a fixed-capacity list (KV-shard wide tier): an empty partial
        if (exporting) {
          int64_t* b = P.w3sum + (int64_t)item * (dv + 1) * (LW + 1);
          for (int64_t i = tid; i < (int64_t)(dv + 1) * (LW + 1); i += T3_THREADS) b[i] = 0;
          if (tid < 4) P.w3max[(int64_t)item * 4 + tid] = tid == 3 ? ST_OK : INT64_MIN;
        }
        continue;  // uniform across the block
      }
      j1 = row_len(P, r);
    }
    // q row
    int qlead = INT32_MIN;
    int qbad = 0;
    for (int i = 0; i < d; ++i) {
      int32_t m, e;
      if (!decode_bf16(P.q[r * d + i], m, e)) qbad = 1;
      if (m) qlead = max(qlead, e + bitlen64((uint64_t)(m < 0 ? -m : m)) - 1);
    }
    const int qlsb = qlead == INT32_MIN ? 0 : qlead + 1 - P.W;
    if (tid == 0) sStatus = qbad ? ST_DOMAIN : ST_OK;
    __syncthreads();

    for (int c0 = 0; c0 < dv; c0 += T3_THREADS) {
      const int c = c0 + tid;
      Wide<LW> Zw, Nw;
      Zw.clear();
      Nw.clear();
      uint64_t Zerr = 0, Nerr = 0;
      int64_t R = INT64_MIN, Emin = INT64_MAX, Emax = INT64_MIN;
      bool has_n = false;
      // sStatus is written only between the top of an iteration and its first barrier, and read
      // only after that barrier, so every thread sees the same value and leaves together.
      for (int64_t t0 = j0; t0 < j1; t0 += T3_THREADS) {
        const int nt = (int)min((int64_t)T3_THREADS, j1 - t0);
        int st = ST_OK;
        int64_t E = 0;
        uint32_t M = 0;
        if (tid < nt) {
          const int64_t kr = key_row(P, r, t0 + tid);
          sRow[tid] = kr;
          const uint16_t* kp = P.k + kr * d;
          int klead = INT32_MIN;
          for (int i = 0; i < d; ++i) {
            int32_t m, e;
            if (!decode_bf16(kp[i], m, e)) st = ST_DOMAIN;
            if (m) klead = max(klead, e + bitlen64((uint64_t)(m < 0 ? -m : m)) - 1);
          }
          const uint16_t* vp = P.v + kr * dv;
          for (int i = 0; i < dv; ++i) {
            int32_t m, e;
            if (!decode_bf16(vp[i], m, e)) st = ST_DOMAIN;
          }
          Rnd t = rnd_zero();
          if (st == ST_OK) {
            const int klsb = klead == INT32_MIN ? 0 : klead + 1 - P.W;
            int64_t acc = 0;
            uint64_t err = 0;
            if (klead != INT32_MIN && qlead != INT32_MIN) {
              for (int i = 0; i < d; ++i) {
                int32_t qm, qe, km, ke;
                decode_bf16(P.q[r * d + i], qm, qe);
                decode_bf16(kp[i], km, ke);
                int ql = 0, kl = 0;
                int32_t qf = qm ? fix_elem(qm, qe, qlsb, ql) : 0;
                int32_t kf = km ? fix_elem(km, ke, klsb, kl) : 0;
                acc += (int64_t)qf * kf;
                err += (uint64_t)ql * (uint64_t)((kf < 0 ? -kf : kf) + kl) + (uint64_t)kl * (uint64_t)(qf < 0 ? -qf : qf);
              }
            }
            int ls = logit_from_interval(acc, err, qlsb + klsb, P.am, P.ae, t);
            if (ls == LOGIT_UNCERTIFIED) {
              ExactScore sc;
              score_clear(sc);
              for (int i = 0; i < d; ++i) {
                int32_t qm, qe, km, ke;
                decode_bf16(P.q[r * d + i], qm, qe);
                decode_bf16(kp[i], km, ke);
                if (qm && km) score_add(sc, qm * km, qe + ke);
              }
              ls = logit_exact(sc, P.am, P.ae, t);
            }
            if (ls == LOGIT_OVERFLOW) st = ST_DOMAIN;
          }
          if (st == ST_OK) {
            int ws = weight_from_logit_wide(t, g_ta128, g_tb128, M, E);
            if (ws == W_HUGE) {
              // integer t with |t| >= 2^30: w = 2^t exactly
              int lead = t.qe + bitlen64(t.q) - 1;
              if (lead >= 62) {
                st = ST_DOMAIN;
              } else {
                int64_t n = (int64_t)(t.q << t.qe);
                M = 1u << 23;
                E = (t.neg ? -n : n) - 23;
              }
            } else if (ws == W_RISKY) {
              st = ST_TIER3;  // unresolved (a 2^-97 event)
            }
          }
          sM[tid] = M;
          sE[tid] = E;
        }
        // block-wide status
        if (st != ST_OK) atomicMax(&sStatus, st);
        __syncthreads();
        const int stc = sStatus;
        if (stc != ST_OK) break;
        const int64_t tmax = block_max64(tid < nt ? sE[tid] + 24 : INT64_MIN, red);
        const int64_t tmin = -block_max64(tid < nt ? -sE[tid] : INT64_MIN, red);
        Emax = max(Emax, tmax - 24);
        Emin = min(Emin, tmin);
        if (Emax - Emin > MAX_SPREAD) {  // uniform: both are block reductions
          if (tid == 0) sStatus = ST_DOMAIN;
          break;
        }
        if (tmax > R) {
          if (R != INT64_MIN) {
            Zw.normalize();
            Nw.normalize();
            int64_t sft = tmax - R;
            bool l1 = Zw.shr(sft), l2 = Nw.shr(sft);
            Zerr = sft >= 64 ? (Zerr != 0) : ((Zerr >> sft) + ((Zerr & ((1ull << sft) - 1)) != 0));
            Nerr = sft >= 64 ? (Nerr != 0) : ((Nerr >> sft) + ((Nerr & ((1ull << sft) - 1)) != 0));
            Zerr += l1;
            Nerr += l2;
          }
          R = tmax;
        }
        for (int jj = 0; jj < nt; ++jj) {
          const int64_t Ej = sE[jj];
          Zw.add((int64_t)sM[jj], Ej - (R - FW), Zerr);
          if (c < dv) {
            int32_t m, e;
            decode_bf16(P.v[sRow[jj] * dv + c], m, e);
            if (m) {
              has_n = true;
              Nw.add((int64_t)sM[jj] * m, Ej + e - (R + 128 - FW), Nerr);
            }
          }
        }
        __syncthreads();
      }
      __syncthreads();
      const int st = sStatus;
      __syncthreads();  // every thread has read sStatus before any finalisation writes it
      if (exporting) {
        // this key range's wide partial (normalised digits), merged across GPUs by
        // wide_rescale_kernel and an all-reduce SUM, finalised by wide_finalize_kernel
        Zw.normalize();
        Nw.normalize();
        int64_t* base = P.w3sum + (int64_t)item * (dv + 1) * (LW + 1);
        if (c0 == 0 && tid == 0) {
          for (int i = 0; i < LW; ++i) base[i] = Zw.d[i];
          base[LW] = (int64_t)Zerr;
          int64_t* mx = P.w3max + (int64_t)item * 4;
          mx[0] = R;
          mx[1] = Emax;
          mx[2] = Emin == INT64_MAX ? INT64_MIN : -Emin;
          mx[3] = st;
        }
        if (c < dv) {
          int64_t* o = base + (int64_t)(1 + c) * (LW + 1);
          for (int i = 0; i < LW; ++i) o[i] = Nw.d[i];
          o[LW] = (int64_t)Nerr;
        }
        __syncthreads();
        continue;
      }
      if (st == ST_OK && c < dv) {
        Rnd res = rnd_zero();
        bool ok = true;
        if (R != INT64_MIN && has_n) {
          Zw.normalize();
          Nw.normalize();
          ok = wide_round(P, Zw, Zerr, Nw, Nerr, res);
        }
        if (ok) {
          write_out(P, r, c, res);
        } else {
          atomicMax(&sStatus, ST_TIER3);
        }
      }
      __syncthreads();
      const int st2 = sStatus;
      __syncthreads();  // read before the next channel block can write it
      if (st2 != ST_OK) break;
    }
    __syncthreads();
    if (exporting) {
      __syncthreads();  // the next row resets sStatus
      continue;
    }
    if (tid == 0) {
      const int st = sStatus;
      if (st == ST_DOMAIN) {
        P.flags[r] = 2;
        stat_add(P, STAT_DOMAIN_ROWS, 1);
      } else if (st == ST_TIER3) {
        P.flags[r] = 1;
        stat_add(P, STAT_UNRESOLVED, 1);
      } else {
        P.flags[r] = 0;
      }
    }
    const int stf = sStatus;
    if (stf == ST_DOMAIN)
      for (int c = tid; c < dv; c += T3_THREADS) write_out(P, r, c, rnd_zero());
    __syncthreads();  // the next row resets sStatus
  }
}

// ---------------------------------------------------------------------------
// wide partials of KV shards (rows tier 1 could not certify after the merge)
// ---------------------------------------------------------------------------
// Thread per (listed row, j): j = 0 is Z, j = 1 + c is channel c's N. The wide windows of every
// shard are shifted down to the merged reference exponent (floor; a dropped nonzero bit and the
// shifted error's ceiling add to the error, as in tier3_kernel's re-anchoring), after which the
// digit-wise SUM over shards is the exact sum of the shards' windows.
__global__ void wide_rescale_kernel(Prob P, int n, const int64_t* gmax) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n * (P.dv + 1)) return;
  const int64_t item = i / (P.dv + 1);
  int64_t* a = P.w3sum + i * (LW + 1);
  const int64_t R = P.w3max[item * 4], G = gmax[item * 4];
  if (R == INT64_MIN) {
    for (int k = 0; k <= LW; ++k) a[k] = 0;
    return;
  }
  if (G <= R) return;
  Wide<LW> w;
  for (int k = 0; k < LW; ++k) w.d[k] = a[k];
  uint64_t err = (uint64_t)a[LW];
  const int64_t sft = G - R;
  const bool lost = w.shr(sft);
  err = sft >= 64 ? (err != 0) : ((err >> sft) + ((err & ((1ull << sft) - 1)) != 0));
  err += lost;
  for (int k = 0; k < LW; ++k) a[k] = w.d[k];
  a[LW] = (int64_t)err;
}

// Certified rounding of one row's merged wide sums (base: Z then every channel's N, digits and
// error; g: merged R, Emax, -Emin, status) into its outputs and flag; a block of T3_THREADS.
__device__ void wide_finalize_row(const Prob& P, const int64_t* base, const int64_t* g, int64_t r, int* sOkp) {
  int& sOk = *sOkp;
  const int tid = threadIdx.x;
  const int64_t R = g[0], Emax = g[1], Emin = g[2] == INT64_MIN ? INT64_MAX : -g[2];
  int st = (int)g[3];
  if (st == ST_OK && R != INT64_MIN && Emax - Emin > MAX_SPREAD) st = ST_DOMAIN;
  if (tid == 0) sOk = 1;
  __syncthreads();
  bool ok = st == ST_OK;
  Wide<LW> Zw;
  uint64_t Zerr = 0;
  if (ok && R != INT64_MIN) {
    for (int k = 0; k < LW; ++k) Zw.d[k] = base[k];
    Zerr = (uint64_t)base[LW];
    Zw.normalize();
  }
  constexpr int CPT = 256 / T3_THREADS;  // dv <= 256
  Rnd res[CPT];
  for (int i = 0; i < CPT; ++i) {
    res[i] = rnd_zero();
    const int c = tid + i * T3_THREADS;
    if (!ok || c >= P.dv || R == INT64_MIN) continue;
    const int64_t* o = base + (int64_t)(1 + c) * (LW + 1);
    Wide<LW> Nw;
    bool any = o[LW] != 0;
    for (int k = 0; k < LW; ++k) {
      Nw.d[k] = o[k];
      any |= o[k] != 0;
    }
    if (!any) continue;
    Nw.normalize();
    ok &= wide_round(P, Zw, Zerr, Nw, (uint64_t)o[LW], res[i]);
  }
  if (st == ST_OK && !ok) atomicAnd(&sOk, 0);
  __syncthreads();
  const bool rowok = st == ST_OK && sOk != 0;
  for (int i = 0; i < CPT; ++i) {
    const int c = tid + i * T3_THREADS;
    if (c < P.dv) write_out(P, r, c, rowok ? res[i] : rnd_zero());
  }
  if (tid == 0) {
    if (st == ST_DOMAIN) {
      P.flags[r] = 2;
      stat_add(P, STAT_DOMAIN_ROWS, 1);
    } else if (!rowok) {
      P.flags[r] = 1;
      stat_add(P, STAT_UNRESOLVED, 1);
    } else {
      P.flags[r] = 0;
    }
  }
}

// Block per listed row: certified rounding of the merged wide sums into the row's outputs.
__global__ void __launch_bounds__(T3_THREADS) wide_finalize_kernel(Prob P, int n, const int64_t* gmax) {
  __shared__ int sOk;
  const int item = blockIdx.x;
  if (item >= n || P.t3_list[item] < 0) return;  // (an unused slot of a fixed-capacity list)
  wide_finalize_row(P, P.w3sum + (int64_t)item * (P.dv + 1) * (LW + 1), gmax + (int64_t)item * 4, P.t3_list[item],
                    &sOk);
}

// Merge of the wide partials in slots first + s * stride (s < cnt) into slot `first` (a block of
// T3_THREADS): MAX of the exponent records, every window floor-shifted to the largest R (the
// error grows by the shift's rounding), digit-wise SUM, as the KV-sharded wide tier does across
// GPUs. The merged record goes to g (which may be the first slot's own record).
__device__ void wide_merge_slots(const Prob& P, int64_t first, int64_t stride, int cnt, int64_t* g, int64_t* red) {
  const int tid = threadIdx.x, dv = P.dv;
  int64_t R = INT64_MIN, Emax = INT64_MIN, nEmin = INT64_MIN, st = ST_OK;
  for (int s = tid; s < cnt; s += T3_THREADS) {
    const int64_t* m = P.w3max + (first + (int64_t)s * stride) * 4;
    R = max(R, m[0]);
    Emax = max(Emax, m[1]);
    nEmin = max(nEmin, m[2]);
    st = max(st, m[3]);
  }
  R = block_max64(R, red);
  Emax = block_max64(Emax, red);
  nEmin = block_max64(nEmin, red);
  st = block_max64(st, red);
  for (int j = tid; j <= dv; j += T3_THREADS) {
    int64_t acc[LW];
    for (int k = 0; k < LW; ++k) acc[k] = 0;
    uint64_t err = 0;
    for (int s = 0; s < cnt; ++s) {
      const int64_t u = first + (int64_t)s * stride;
      const int64_t Ru = P.w3max[u * 4];
      if (Ru == INT64_MIN) continue;  // no keys in this slot
      const int64_t* a = P.w3sum + (u * (dv + 1) + j) * (LW + 1);
      Wide<LW> w;
      for (int k = 0; k < LW; ++k) w.d[k] = a[k];
      uint64_t e = (uint64_t)a[LW];
      if (R > Ru) {
        const int64_t sft = R - Ru;
        const bool lost = w.shr(sft);
        e = sft >= 64 ? (e != 0) : ((e >> sft) + ((e & ((1ull << sft) - 1)) != 0));
        e += lost;
      }
      for (int k = 0; k < LW; ++k) acc[k] += w.d[k];
      err += e;
    }
    int64_t* o = P.w3sum + (first * (dv + 1) + j) * (LW + 1);
    for (int k = 0; k < LW; ++k) o[k] = acc[k];
    o[LW] = (int64_t)err;
  }
  __syncthreads();  // every slot's record and windows have been read
  if (tid == 0) {
    g[0] = R;
    g[1] = Emax;
    g[2] = nEmin;
    g[3] = st;
  }
  __syncthreads();
}

// Level 1 of the tier-3 merge (split mode only): block per group head of T3_GROUP units, merged in
// place into the head's slot; the digit sums are renormalised before level 2 adds them up again.
__global__ void __launch_bounds__(T3_THREADS) tier3_group_kernel(Prob P) {
  __shared__ int64_t red[T3_THREADS / 32];
  if (P.u_n[3] != 0) return;
  const int n = (int)P.u_n[0], dv = P.dv;
  const int64_t units = P.u_n[1];
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int i = unit_row(P.u_off, n, u);
    if ((u - P.u_off[i]) % T3_GROUP != 0) continue;  // uniform across the block
    const int cnt = (int)min((int64_t)T3_GROUP, (int64_t)P.u_off[i + 1] - u);
    wide_merge_slots(P, u, 1, cnt, P.w3max + u * 4, red);
    // normalise the head's windows (each digit back to 32 bits) for the next level's shifts
    for (int j = threadIdx.x; j <= dv; j += T3_THREADS) {
      int64_t* a = P.w3sum + (u * (dv + 1) + j) * (LW + 1);
      if (P.w3max[u * 4] == INT64_MIN) continue;
      Wide<LW> w;
      for (int k = 0; k < LW; ++k) w.d[k] = a[k];
      w.normalize();
      for (int k = 0; k < LW; ++k) a[k] = w.d[k];
    }
    __syncthreads();
  }
}

// Tier-3 merge of a split-K run, level 2 (nothing to do in whole-row mode): block per planned row,
// its group heads merged into its first slot, then certified. g3: merged records (T3_SPLIT_ROWS x 4).
__global__ void __launch_bounds__(T3_THREADS) tier3_merge_kernel(Prob P, int64_t* g3) {
  __shared__ int64_t red[T3_THREADS / 32];
  __shared__ int sOk;
  if (P.u_n[3] != 0) return;
  const int n = (int)P.u_n[0], tid = threadIdx.x, dv = P.dv;
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int u0 = P.u_off[i], u1 = P.u_off[i + 1];
    int64_t* g = g3 + (int64_t)i * 4;
    wide_merge_slots(P, u0, T3_GROUP, (u1 - u0 + T3_GROUP - 1) / T3_GROUP, g, red);
    wide_finalize_row(P, P.w3sum + (int64_t)u0 * (dv + 1) * (LW + 1), g, P.u_rows[i], &sOk);
    __syncthreads();
    (void)tid;
  }
}

// ---------------------------------------------------------------------------
// launchers (called from ea_api.cu)
// ---------------------------------------------------------------------------
template <int CPL>
static cudaError_t launch_simt_cpl(const Prob& P, int warps, cudaStream_t st) {
  size_t smem = simt_smem_bytes(P.d, P.dv, warps);
  cudaError_t e = cudaFuncSetAttribute(simt_split_kernel<CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((P.rows + warps - 1) / warps), (unsigned)P.splits);
  simt_split_kernel<CPL><<<grid, warps * 32, smem, st>>>(P);
  e = cudaGetLastError();
  if (e != cudaSuccess || P.splits == 1) return e;
  combine_kernel<CPL><<<(unsigned)((P.rows + 3) / 4), 128, 0, st>>>(P);
  return cudaGetLastError();
}

int simt_warps_for(int d, int dv) {
  int w = 4;
  while (w > 1 && simt_smem_bytes(d, dv, w) > 200 * 1024) --w;
  return w;
}

cudaError_t launch_simt(const Prob& P, cudaStream_t st) {
  int warps = simt_warps_for(P.d, P.dv);
  if (P.dv <= 32) return launch_simt_cpl<1>(P, warps, st);
  if (P.dv <= 64) return launch_simt_cpl<2>(P, warps, st);
  if (P.dv <= 128) return launch_simt_cpl<4>(P, warps, st);
  return launch_simt_cpl<8>(P, warps, st);
}

cudaError_t launch_combine(const Prob& P, cudaStream_t st) {
  const unsigned g = (unsigned)((P.rows + 3) / 4);
  if (P.dv <= 128 && P.rows <= 0x7FFFFFFF) combine_row_kernel<<<(unsigned)P.rows, 128, 0, st>>>(P);
  else if (P.dv <= 32) combine_kernel<1><<<g, 128, 0, st>>>(P);
  else if (P.dv <= 64) combine_kernel<2><<<g, 128, 0, st>>>(P);
  else if (P.dv <= 128) combine_kernel<4><<<g, 128, 0, st>>>(P);
  else combine_kernel<8><<<g, 128, 0, st>>>(P);
  return cudaGetLastError();
}

cudaError_t launch_partials_rescale(const Prob& P, const int32_t* Rg, const int32_t* NRg, cudaStream_t st) {
  const int64_t n = P.rows * P.dv;
  partials_rescale_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(P, Rg, NRg);
  return cudaGetLastError();
}

cudaError_t launch_partials_finalize(const Prob& P, cudaStream_t st) {
  const unsigned g = (unsigned)((P.rows + 3) / 4);
  if (P.dv <= 32) partials_finalize_kernel<1><<<g, 128, 0, st>>>(P);
  else if (P.dv <= 64) partials_finalize_kernel<2><<<g, 128, 0, st>>>(P);
  else if (P.dv <= 128) partials_finalize_kernel<4><<<g, 128, 0, st>>>(P);
  else partials_finalize_kernel<8><<<g, 128, 0, st>>>(P);
  return cudaGetLastError();
}

cudaError_t launch_wide_rescale(const Prob& P, int n, const int64_t* gmax, cudaStream_t st) {
  const int64_t m = (int64_t)n * (P.dv + 1);
  wide_rescale_kernel<<<(unsigned)((m + 127) / 128), 128, 0, st>>>(P, n, gmax);
  return cudaGetLastError();
}

cudaError_t launch_wide_finalize(const Prob& P, int n, const int64_t* gmax, cudaStream_t st) {
  wide_finalize_kernel<<<n, T3_THREADS, 0, st>>>(P, n, gmax);
  return cudaGetLastError();
}

// Every row on the tier-3 list (value rows wider than the tier-1 kernels take), with the pair count.
__global__ void list_all_rows_kernel(Prob P) {
  __shared__ unsigned long long pairs;
  if (threadIdx.x == 0) pairs = 0;
  __syncthreads();
  unsigned long long mine = 0;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < P.rows; r += (int64_t)gridDim.x * blockDim.x) {
    P.t3_list[r] = (int)r;
    mine += (unsigned long long)row_len(P, r);
  }
  atomicAdd(&pairs, mine);
  __syncthreads();
  if (threadIdx.x == 0) {
    stat_add(P, STAT_PAIRS, pairs);
    if (blockIdx.x == 0) *P.t3_count = (int)P.rows;
  }
}

cudaError_t launch_list_all_rows(const Prob& P, cudaStream_t st) {
  const int64_t b = (P.rows + 255) / 256;
  list_all_rows_kernel<<<(unsigned)(b < 1024 ? b : 1024), 256, 0, st>>>(P);
  return cudaGetLastError();
}

cudaError_t launch_tier3(const Prob& P, int blocks, cudaStream_t st) {
  tier3_kernel<<<blocks, T3_THREADS, 0, st>>>(P);
  return cudaGetLastError();
}

size_t fallback_bytes(int dv) {
  auto a = [](size_t x) { return (x + 255) & ~(size_t)255; };
  return a((T2_MAX_ROWS + 1) * 4) + a((T3_SPLIT_ROWS + 1) * 4) + 2 * a(4 * 8) + a((size_t)T3_SPLIT_ROWS * 4 * 8) +
         3 * a((size_t)T2_UNITS * 4) + 2 * a((size_t)T2_UNITS * 8) + a((size_t)T2_UNITS * dv * 4) +
         2 * a((size_t)T2_UNITS * dv * 8) + a((size_t)T3_UNITS * 4 * 8) + a((size_t)T3_UNITS * (dv + 1) * (LW + 1) * 8);
}

// carves a fallback_bytes(dv) block into the fallback buffers (list3 / count3 come separately)
void fallback_carve(void* base, int dv, FallbackBufs& F) {
  char* p = (char*)base;
  auto take = [&](size_t bytes) {
    char* r = p;
    p += (bytes + 255) & ~(size_t)255;
    return (void*)r;
  };
  F.u2_off = (int*)take((T2_MAX_ROWS + 1) * 4);
  F.u3_off = (int*)take((T3_SPLIT_ROWS + 1) * 4);
  F.u2_n = (int64_t*)take(4 * 8);
  F.u3_n = (int64_t*)take(4 * 8);
  F.g3 = (int64_t*)take((size_t)T3_SPLIT_ROWS * 4 * 8);
  F.pR = (int32_t*)take((size_t)T2_UNITS * 4);
  F.pSt = (int32_t*)take((size_t)T2_UNITS * 4);
  F.pRlo = (int32_t*)take((size_t)T2_UNITS * 4);
  F.pZ = (int64_t*)take((size_t)T2_UNITS * 8);
  F.pZe = (uint64_t*)take((size_t)T2_UNITS * 8);
  F.pNR = (int32_t*)take((size_t)T2_UNITS * dv * 4);
  F.pN = (int64_t*)take((size_t)T2_UNITS * dv * 8);
  F.pNe = (uint64_t*)take((size_t)T2_UNITS * dv * 8);
  F.w3max = (int64_t*)take((size_t)T3_UNITS * 4 * 8);
  F.w3sum = (int64_t*)take((size_t)T3_UNITS * (dv + 1) * (LW + 1) * 8);
}

template <int CPL>
static cudaError_t launch_tier2_cpl(const Prob& P2, int32_t* pRlo, int sms, cudaStream_t st) {
  const int warps = simt_warps_for(P2.d, P2.dv);
  const size_t smem = simt_smem_bytes(P2.d, P2.dv, warps);
  cudaError_t e = cudaFuncSetAttribute(tier2_units_kernel<CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int gu = min((T2_UNITS + warps - 1) / warps, 4 * sms);
  tier2_units_kernel<CPL><<<gu, warps * 32, smem, st>>>(P2);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  tier2_group_kernel<CPL><<<min(T2_UNITS / 4, 4 * sms), 128, 0, st>>>(P2, pRlo);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  tier2_merge_kernel<CPL><<<min(T2_MAX_ROWS / 4, 2 * sms), 128, 0, st>>>(P2, pRlo);
  return cudaGetLastError();
}

// The fallback tiers after a tier-1 launch of P (dv <= 256): tier 2 reruns the rows tier 1
// listed (P.t3_list, *P.t3_count), tier 3 computes what tier 2 could not certify (split by key
// chunks when few rows are left). Fixed launches that read their work from device memory, so
// nothing waits on the host and the sequence can be captured in a CUDA graph.
cudaError_t launch_fallback(const Prob& P, const FallbackBufs& F, int sms, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(F.count3, 0, sizeof(int), st);
  if (e != cudaSuccess) return e;
  fallback_plan_kernel<<<1, 1024, 0, st>>>(P, P.t3_list, P.t3_count, T2_MAX_ROWS, T2_UNITS, T2_MIN_CHUNK, F.u2_off,
                                           F.u2_n, F.list3, F.count3, 0);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  Prob P2 = P;
  P2.tier = 2;
  P2.splits = 1;
  P2.export_partials = 0;
  P2.t3_fixed = 0;
  P2.u_off = F.u2_off;
  P2.u_n = F.u2_n;
  P2.u_rows = P.t3_list;
  P2.t3_list = F.list3;
  P2.t3_count = F.count3;
  P2.pR = F.pR;
  P2.pZ = F.pZ;
  P2.pZe = F.pZe;
  P2.pSt = F.pSt;
  P2.pNR = F.pNR;
  P2.pN = F.pN;
  P2.pNe = F.pNe;
  if (P.dv <= 32) e = launch_tier2_cpl<1>(P2, F.pRlo, sms, st);
  else if (P.dv <= 64) e = launch_tier2_cpl<2>(P2, F.pRlo, sms, st);
  else if (P.dv <= 128) e = launch_tier2_cpl<4>(P2, F.pRlo, sms, st);
  else e = launch_tier2_cpl<8>(P2, F.pRlo, sms, st);
  if (e != cudaSuccess) return e;
  fallback_plan_kernel<<<1, 1024, 0, st>>>(P, F.list3, F.count3, T3_SPLIT_ROWS, T3_UNITS, T3_MIN_CHUNK, F.u3_off,
                                           F.u3_n, nullptr, nullptr, 1);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  Prob P3 = P;
  P3.tier = 3;
  P3.export_partials = 0;
  P3.t3_fixed = 0;
  P3.u_off = F.u3_off;
  P3.u_n = F.u3_n;
  P3.u_rows = F.list3;
  P3.w3max = F.w3max;
  P3.w3sum = F.w3sum;
  tier3_kernel<<<2 * sms, T3_THREADS, 0, st>>>(P3);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  tier3_group_kernel<<<min(T3_UNITS, 2 * sms), T3_THREADS, 0, st>>>(P3);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  tier3_merge_kernel<<<min(T3_SPLIT_ROWS, 2 * sms), T3_THREADS, 0, st>>>(P3, F.g3);
  return cudaGetLastError();
}

}  // namespace ea
