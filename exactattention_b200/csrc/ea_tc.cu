// Tensor-core (tcgen05 / TMEM) tier-1 kernel of certified ExactAttention for row blocks that share
// a contiguous key range (causal / prefix prefill): d = dv = 128, 128 rows per CTA, 64-key tiles,
// 512 threads. Thread (row r = 32 (warp % 4) + lane, quarter u = warp / 4) owns TMEM lane r, keys
// 16u .. 16u + 15 of every tile and channels 32u .. 32u + 31 of the row's running sums.
//
// Exactness (all integer):
//   scores   q and k rows in block fixed point (W bits, two's complement) cut into 4 byte digits
//            (low three unsigned, top signed); S = sum_(s,t) 2^(8(s+t)) Q_s . K_t with the 16 digit
//            products grouped by s + t into 7 int32 TMEM accumulators (each |.| < 2^25), recombined
//            in int64 (|S| < 2^61). The truncation bound err is summed over the lossy elements
//            only; t = RN32(alpha S) is certified at both ends, else the exact score (a 128-bit
//            window over the pair's products, or 576-bit bins when they span more) decides, one
//            warp per pair.
//   weights  RN24(2^t) by the integer exp2; W = floor(w / 2^(Rt - 48)) (Rt: the row's tile bound
//            max ceil(t) + 1 >= max floor(t) + 2 > log2 w, so W < 2^48) cut into 6 unsigned bytes.
//   P.V      v in fixed point against the largest |v| exponent VE_c of each channel over the
//            block's keys, |Vfix| < 2^23, 3 byte digits; sum_j W Vfix = sum_g 2^(8g) D_g with the
//            18 digit products grouped into 8 int32 accumulators (|.| < 2^24), each shifted into the
//            running int64 N (units 2^(R + VE_c - FN)); the floor of a right shift costs one unit.
//   bounds   per row, in units of each channel's own N unit: truncated weights (< 1 W unit times
//            |v| < 2^VE_c), truncated values (keys flagged lossy), shift floors and rescales.
//            Z is exact up to counted truncations. The final N/Z interval is certified per channel;
//            a row with any uncertified channel, a huge logit or a still-risky weight goes to tier 3.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ea_core.cuh"
#include "ea_fast64.cuh"
#include "ea_numerics.h"
#include "ea_tables.cuh"
#include "ea_tc_common.cuh"
#include "ea_tcgen05.cuh"

namespace ea {

namespace tck {

using namespace tcc;

constexpr int BM = 128, BN = 64, D = 128, DV = 128;
constexpr int NQ = 4, NK = 4, NW = 6, NV = 3;
constexpr int NGS = NQ + NK - 1;  // score groups
constexpr int NGP = NW + NV - 1;  // P.V groups
constexpr int FW = 48, FV = 23;
constexpr int THREADS = 512, NWARPS = THREADS / 32;
constexpr int LCAP = 4;  // window elements per q row / key whose lost parts are kept for the correction
constexpr uint32_t TMEM_COLS = 512;

// shared memory map (bytes)
constexpr uint32_t Q_PLANE = BM * D;         // 16384
// K planes: the 16-byte K chunks of the 64 keys 1040 bytes apart (LBO), not 1024, so the 8 chunks
// of one key row that a quarter warp stores land in 8 different bank groups
constexpr uint32_t KLBO = (BN / 8) * 128 + 16;  // 1040
constexpr uint32_t K_PLANE = (D / 16) * KLBO;   // 8320
constexpr uint32_t V_PLANE = DV * BN;        // 8192
constexpr uint32_t W_PLANE = BM * BN;        // 8192
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + NQ * Q_PLANE;
constexpr uint32_t OFF_V = OFF_K + NK * K_PLANE;
constexpr uint32_t OFF_W = OFF_V + NV * V_PLANE;
constexpr uint32_t T_PITCH = BN + 1;
constexpr uint32_t OFF_T = OFF_W + NW * W_PLANE;
constexpr uint32_t OFF_SMALL = OFF_T + BM * T_PITCH * 4;

struct Small {
  int32_t rows[BM];
  int32_t len[BM];
  int32_t qlsb[BM];
  uint32_t qlossy[BM][4];
  int32_t rst[BM];        // row status
  int32_t rok[BM];        // all channels certified
  int32_t rt[4][BM];      // tile bound exchange
  uint32_t zl[4][BM];     // lossy weights exchange
  uint64_t zs[4][BM];     // tile Z exchange
  uint64_t vw[4][BM];     // sum of W + 1 over keys with lossy values
  int32_t klsb[BN];
  uint32_t klossy[BN][4];
  int32_t kbad[BN];
  int32_t vlossy[BN];
  uint32_t kmeta[BN];  // per key, for pass 1: klsb (low 16 bits, signed) | lossy << 16 | bad << 17
  // the window elements of each q row (key of the tile) that lost bits, up to LCAP, with their
  // lost parts dq = q - Q 2^qlsb (dk = k - K 2^klsb): at most 8 significant bits at or above the
  // bf16 subnormal unit 2^-133, so exact in fp32; count > LCAP: the list is incomplete
  float qc_d[BM][LCAP];
  float kc_d[BN][LCAP];
  uint8_t qc_i[BM][LCAP];
  uint8_t kc_i[BN][LCAP];
  uint8_t qc_n[BM];
  uint8_t kc_n[BN];
  int32_t ve[DV];
  uint64_t td[256];  // binary64 2^(j/256) of the fast weight path
  uint64_t bar;        // score MMAs
  uint64_t bar_pv[2];  // P.V rounds, by round parity
  uint32_t tmem;
  int32_t maxlen;
  int32_t ka, kb;  // this KV split's keys of the block's range
  int64_t base;
};

constexpr uint32_t SMEM_BYTES = OFF_SMALL + sizeof(Small);
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

#ifdef EA_PHASE_TIMERS
__device__ unsigned long long g_phase_cycles[16];
#endif

// byte offset of (key j, byte k) in a K digit plane (the K-major layout with the padded LBO)
__device__ __forceinline__ uint32_t koff(uint32_t j, uint32_t k) {
  return (k >> 4) * KLBO + (j >> 3) * 128u + (j & 7u) * 16u + (k & 15u);
}
// int32 fixed-point value of key j's element k from the K digit planes
__device__ __forceinline__ int32_t read_fix_k(const uint8_t* sK, uint32_t j, uint32_t k) {
  const uint32_t o = koff(j, k);
  const uint32_t b0 = sK[o], b1 = sK[o + K_PLANE], b2 = sK[o + 2 * K_PLANE];
  const int32_t b3 = (int8_t)sK[o + 3 * K_PLANE];
  return (int32_t)(b0 | (b1 << 8) | (b2 << 16)) + (b3 << 24);
}

// Truncation bound of one windowed score, in units 2^(qlsb + klsb): for the lossy elements only,
// |q k - Q K| <= |dq| |k| + |Q| |dk| with |dq|, |dk| < 1 unit and |k| < |K| + 1 unit when k is lossy.
__device__ __noinline__ uint64_t score_err(const Small& S, const uint8_t* sQ, const uint8_t* sK, int r, int kj) {
  uint64_t err = 0;
  for (int w = 0; w < 4; ++w) {
    const uint32_t ql = S.qlossy[r][w], kl = S.klossy[kj][w];
    for (uint32_t m = ql; m; m &= m - 1) {
      int i = 32 * w + __ffs(m) - 1;
      int32_t kf = read_fix_k(sK, kj, i);
      err += (uint64_t)(kf < 0 ? -kf : kf) + ((kl >> (i & 31)) & 1u);
    }
    for (uint32_t m = kl; m; m &= m - 1) {
      int i = 32 * w + __ffs(m) - 1;
      int32_t qf = read_fix(sQ, Q_PLANE, r, i, BM);
      err += (uint64_t)(qf < 0 ? -qf : qf);
    }
  }
  return err;
}

// The exact correction of one windowed score for its lossy elements, in binary64: with
// q = Q 2^qlsb + dq and k = K 2^klsb + dk (dq, dk: the parts truncation dropped, exact),
// q k - Q K 2^(qlsb + klsb) = Q 2^qlsb dk + dq k, one rounding per element (an fma of exact
// products), then a sum of n terms: |corr - c| <= (n + 1) 2^-53 sum |terms| (returned in err).
__device__ __noinline__ double score_corr(const Small& S, const uint8_t* sQ, const uint8_t* sK, int r, int kj,
                                          const uint16_t* qrow, const uint16_t* krow, int qlsb, int klsb,
                                          double& err) {
  const double pq = __hiloint2double((qlsb + 1023) << 20, 0), pk = __hiloint2double((klsb + 1023) << 20, 0);
  double c = 0.0, a = 0.0;
  int n = 0;
  for (int w = 0; w < 4; ++w) {
    for (uint32_t m = S.qlossy[r][w] | S.klossy[kj][w]; m; m &= m - 1) {
      const int i = 32 * w + __ffs(m) - 1;
      // a bf16 is exact as the fp32 with its bits on top, and so in binary64
      const double q = (double)__uint_as_float((uint32_t)qrow[i] << 16);
      const double k = (double)__uint_as_float((uint32_t)krow[i] << 16);
      const double Qs = (double)read_fix(sQ, Q_PLANE, r, i, BM) * pq;
      const double Ks = (double)read_fix_k(sK, kj, i) * pk;
      const double t = __fma_rn(Qs, k - Ks, (q - Qs) * k);
      c += t;
      a += fabs(t);
      ++n;
    }
  }
  err = (double)(n + 2) * 1.1102230246251565e-16 * a * 1.000001;
  return c;
}

// As score_corr, from the per-row and per-key lists of lost parts kept in shared memory (no
// global loads): for an element lossy in q only, the term is dq k with k = K 2^klsb exact; for one
// lossy in k only, Q 2^qlsb dk (exact); for one lossy in both, Q 2^qlsb dk + dq k (one rounding).
// False when a list is incomplete.
__device__ __forceinline__ bool score_corr_cached(const Small& S, const uint8_t* sQ, const uint8_t* sK, int r, int kj,
                                                  int qlsb, int klsb, double& corr, double& err) {
  const int nq = S.qc_n[r], nk = S.kc_n[kj];
  if (nq > LCAP || nk > LCAP) return false;
  const double pq = __hiloint2double((qlsb + 1023) << 20, 0), pk = __hiloint2double((klsb + 1023) << 20, 0);
  double c = 0.0, a = 0.0;
  for (int e = 0; e < nq; ++e) {
    const int i = S.qc_i[r][e];
    double dk = 0.0;
    for (int f = 0; f < nk; ++f)
      if (S.kc_i[kj][f] == i) dk = (double)S.kc_d[kj][f];
    const double k = (double)read_fix_k(sK, kj, i) * pk + dk;  // the element itself, exact
    const double Qs = dk != 0.0 ? (double)read_fix(sQ, Q_PLANE, r, i, BM) * pq : 0.0;
    const double t = __fma_rn(Qs, dk, (double)S.qc_d[r][e] * k);
    c += t;
    a += fabs(t);
  }
  for (int f = 0; f < nk; ++f) {
    const int i = S.kc_i[kj][f];
    bool inq = false;
    for (int e = 0; e < nq; ++e) inq |= S.qc_i[r][e] == i;
    if (inq) continue;
    const double t = (double)read_fix(sQ, Q_PLANE, r, i, BM) * pq * (double)S.kc_d[kj][f];  // exact
    c += t;
    a += fabs(t);
  }
  corr = c;
  err = (double)(nq + nk + 2) * 1.1102230246251565e-16 * a * 1.000001;
  return true;
}

__global__ void __launch_bounds__(THREADS, 1) tc_prefill_kernel(Prob P, const int32_t* __restrict__ block_rows) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sQ = smem + OFF_Q;
  uint8_t* sK = smem + OFF_K;
  uint8_t* sV = smem + OFF_V;
  uint8_t* sW = smem + OFF_W;
  uint32_t* sT = (uint32_t*)(smem + OFF_T);
  Small& S = *(Small*)(smem + OFF_SMALL);
  EA_PT_DECL

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int blk = blockIdx.x;

  // ---------------- set-up ----------------
  if (tid < BM) {
    int32_t row = block_rows[(int64_t)blk * BM + tid];
    S.rows[tid] = row;
    S.len[tid] = row >= 0 ? (int32_t)P.kv_len[row] : 0;
    S.rst[tid] = ST_OK;
    S.rok[tid] = 1;
  }
  if (tid < 256) S.td[tid] = f64::g_exp2_d64[tid];
  if (tid == 0) {
    tc::mbar_init(&S.bar, NGS);        // one commit per score group's issuer
    tc::mbar_init(&S.bar_pv[0], 2);    // one commit per P.V group's issuer (two groups a round)
    tc::mbar_init(&S.bar_pv[1], 2);
    S.base = P.kv_base[block_rows[(int64_t)blk * BM]];
  }
  if (warp == 0) tc::tmem_alloc(&S.tmem, TMEM_COLS);
  __syncthreads();
  if (tid == 0) {
    int32_t m = 0;
    for (int i = 0; i < BM; ++i) m = max(m, S.len[i]);
    // KV split blockIdx.y of gridDim.y: keys [ka, kb) of the block's range, the cut points
    // rounded down to whole tiles; every row keeps its keys below kb, from ka on
    int32_t ka = 0, kb = m;
    if (gridDim.y > 1) {
      const int64_t sp = blockIdx.y, ns = gridDim.y;
      ka = (int32_t)(((int64_t)m * sp / ns) & ~(int64_t)(BN - 1));
      kb = sp + 1 == ns ? m : (int32_t)(((int64_t)m * (sp + 1) / ns) & ~(int64_t)(BN - 1));
      S.base += ka;
      m = max(0, kb - ka);
    }
    S.ka = ka;
    S.kb = kb;
    S.maxlen = m;
  }
  if (gridDim.y > 1) {
    __syncthreads();
    if (tid < BM) S.len[tid] = max(0, min(S.len[tid], S.kb) - S.ka);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = S.tmem;
  const int32_t maxlen = S.maxlen;
  const int64_t base = S.base;

  // q rows -> 4 digit planes; thread (row tid / 4, quarter tid % 4) converts 32 elements
  {
    const int i = tid >> 2, qq = tid & 3;
    const int32_t row = S.rows[i];
    uint32_t bits[32];
    int lead = INT32_MIN, bad = 0;
    if (row >= 0) {
      const uint4* src = (const uint4*)(P.q + (int64_t)row * D + 32 * qq);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 x = src[c];
        const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          bits[8 * c + 2 * u] = w4[u] & 0xFFFFu;
          bits[8 * c + 2 * u + 1] = w4[u] >> 16;
        }
      }
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        int32_t m, ex;
        if (!decode_bf16(bits[e], m, ex)) bad = 1;
        if (m) lead = max(lead, lead_of(m, ex));
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) bits[e] = 0;
    }
    lead = max(lead, __shfl_xor_sync(0xffffffffu, lead, 1));
    lead = max(lead, __shfl_xor_sync(0xffffffffu, lead, 2));
    bad |= __shfl_xor_sync(0xffffffffu, bad, 1);
    bad |= __shfl_xor_sync(0xffffffffu, bad, 2);
    const int lsb = lead == INT32_MIN ? 0 : lead + 1 - P.W;
    uint32_t lmask = 0;
    uint32_t x[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      int lost = 0, b2 = 0;
      x[e] = (bad || lead == INT32_MIN) ? 0u : (uint32_t)fixq(bits[e], lsb, lost, b2);
      if (lost) lmask |= 1u << e;
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint4 pl[NQ];
      planes16<NQ>(x + 16 * c, pl);
#pragma unroll
      for (int p = 0; p < NQ; ++p) *(uint4*)(sQ + p * Q_PLANE + tc::kmajor_off(i, 32 * qq + 16 * c, BM)) = pl[p];
    }
    S.qlossy[i][qq] = lmask;
    if (qq == 0) {
      S.qlsb[i] = lsb;
      if (bad && row >= 0) S.rst[i] = ST_DOMAIN;
    }
  }
  // channel exponents over the block's keys: VE_c = max (lead(v) + 1) over the finite values, or
  // INT32_MIN if all are zero. Thread: 16-byte piece q = tid % 16 (channels 8q .. 8q + 7) of keys
  // tid / 16, + 32, ..; NaN / inf values are caught per tile.
  {
    const int q = tid & 15;
    uint32_t mx[4] = {0u, 0u, 0u, 0u};
#pragma unroll 4
    for (int64_t j = tid >> 4; j < maxlen; j += THREADS / 16) {
      const uint4 x = *(const uint4*)(P.v + (base + j) * DV + 8 * q);
      mx[0] = __vmaxu2(mx[0], x.x & 0x7FFF7FFFu);
      mx[1] = __vmaxu2(mx[1], x.y & 0x7FFF7FFFu);
      mx[2] = __vmaxu2(mx[2], x.z & 0x7FFF7FFFu);
      mx[3] = __vmaxu2(mx[3], x.w & 0x7FFF7FFFu);
    }
    // a channel that saw a NaN / inf: its largest finite magnitude, rescanned (rare)
    if (__vcmpgeu2(__vmaxu2(__vmaxu2(mx[0], mx[1]), __vmaxu2(mx[2], mx[3])), 0x7F807F80u)) {
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        if (((mx[h >> 1] >> (16 * (h & 1))) & 0xFFFFu) < 0x7F80u) continue;
        uint32_t m = 0;
        for (int64_t j = tid >> 4; j < maxlen; j += THREADS / 16) {
          const uint32_t e = P.v[(base + j) * DV + 8 * q + h] & 0x7FFFu;
          if (e < 0x7F80u) m = max(m, e);
        }
        mx[h >> 1] = (mx[h >> 1] & ~(0xFFFFu << (16 * (h & 1)))) | (m << (16 * (h & 1)));
      }
    }
    uint32_t* part = sT;  // [16 warps][128 channels], free until the first tile's pass 1
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t o = __vmaxu2(mx[w], __shfl_xor_sync(0xffffffffu, mx[w], 16));  // keys of the other half-warp
      if (lane < 16) {
        part[warp * DV + 8 * q + 2 * w] = o & 0xFFFFu;
        part[warp * DV + 8 * q + 2 * w + 1] = o >> 16;
      }
    }
    __syncthreads();
    if (tid < DV) {
      uint32_t m = 0;
#pragma unroll
      for (int w = 0; w < NWARPS; ++w) m = max(m, part[w * DV + tid]);
      S.ve[tid] = m == 0 ? INT32_MIN : lead_of_bits(m) + 1;
    }
    __syncthreads();
  }

  // the q rows' lists of lost window parts (the planes and the lossy masks are complete here)
  if (tid < BM) {
    const int32_t row = S.rows[tid];
    const int qlsb = S.qlsb[tid];
    const double pq = __hiloint2double((qlsb + 1023) << 20, 0);
    int n = 0;
    for (int w = 0; w < 4; ++w)
      for (uint32_t m = S.qlossy[tid][w]; m; m &= m - 1) {
        const int i = 32 * w + __ffs(m) - 1;
        if (n < LCAP) {
          const double q = (double)__uint_as_float((uint32_t)P.q[(int64_t)row * D + i] << 16);
          S.qc_d[tid][n] = (float)(q - (double)read_fix(sQ, Q_PLANE, tid, i, BM) * pq);  // exact
          S.qc_i[tid][n] = (uint8_t)i;
        }
        ++n;
      }
    S.qc_n[tid] = (uint8_t)min(n, 255);
  }
  __syncthreads();

  EA_PT_INIT
  const int r = 32 * (warp & 3) + lane, u4 = warp >> 2;
  const uint32_t tlane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
  const int32_t myrow = S.rows[r];
  const int32_t mylen = S.len[r];
  const int FN = P.FZ, FZ = P.FZ;
  int32_t R = R_EMPTY;
  int64_t Z = 0;
  uint64_t Zerr = 0, Nerr = 0;
  int64_t N[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) N[c] = 0;
  uint32_t phase = 0;
  float tlo = INFINITY;  // this thread's lowest certified logit (the exponent-spread check)
  uint32_t pv_phase = 0, pv_pending = 0;  // P.V barriers: phase bits, commits in flight (by parity)
  bool ok_wait = true;
  unsigned n_exact = 0, n_wide = 0;
  const double am_d = (double)P.am;

  for (int32_t j0 = 0; j0 < maxlen; j0 += BN) {
    // ---------------- K tile -> digit planes (thread: key tid / 8, elements 16 (tid % 8) ..) --------
    // The block exponent comes from the key's largest |k|. When no nonzero element lies below the
    // window (smallest nonzero |k| has an exponent field >= ebase), every element converts exactly
    // through fp32 (x = trunc(k 2^-lsb), |x| < 2^W); otherwise element by element with loss flags.
    {
      const int j = tid >> 3, e8 = tid & 7;
      const bool valid = j0 + j < maxlen;
      uint32_t w[8];
      if (valid) {
        const uint4* src = (const uint4*)(P.k + (base + j0 + j) * D + 16 * e8);
        const uint4 a = src[0], b = src[1];
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
        w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = 0u;
      }
      uint32_t mx = 0, mk = NZ_NONE;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t m = w[i] & 0x7FFF7FFFu;
        mx = __vmaxu2(mx, m);
        mk = __vmins2(mk, nz_key(m));
      }
      mx = max(mx & 0xFFFFu, mx >> 16);
      int32_t mn = nz_key_min(mk);
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      }
      const int bad = mx >= 0x7F80u;
      const int lead = (mx == 0 || bad) ? INT32_MIN : lead_of_bits(mx);
      const int lsb = lead == INT32_MIN ? 0 : lead + 1 - P.W;
      const int ebase = lsb + 134;  // an element with exponent field E >= ebase loses no bits
      const bool fast = lead == INT32_MIN || (lsb >= -126 && lsb <= 126 &&
                                              (mn == 32767 || nz_key_mag(mn) >= ((uint32_t)ebase << 7)));
      uint32_t lmask = 0;
      uint32_t x[16];
      if (lead == INT32_MIN) {
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = 0u;
      } else if (fast) {
        const float sc = scale_of(lsb);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          x[2 * i] = fixf_lo(w[i], sc);
          x[2 * i + 1] = fixf_hi(w[i], sc);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          int lost = 0, b2 = 0;
          x[e] = (uint32_t)fixq((w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu, lsb, lost, b2);
          if (lost) lmask |= 1u << e;
        }
      }
      uint4 pl[NK];
      planes16<NK>(x, pl);
#pragma unroll
      for (int p = 0; p < NK; ++p) *(uint4*)(sK + p * K_PLANE + koff(j, 16 * e8)) = pl[p];
      const uint32_t other = __shfl_xor_sync(0xffffffffu, lmask, 1);
      if ((e8 & 1) == 0) S.klossy[j][e8 >> 1] = lmask | (other << 16);
      if (e8 == 0) {
        S.klsb[j] = lsb;
        S.kbad[j] = valid && bad;
        S.vlossy[j] = 0;
      }
    }
    tc::fence_async_smem();
    __syncthreads();
    EA_PT(0)
    // the keys' lists of lost window parts (threads 64 .. 127; read in pass 1, after the next barrier)
    if (tid >= 64 && tid < 64 + BN) {
      const int jj = tid - 64;
      const int klsb = S.klsb[jj];
      const double pk = __hiloint2double((klsb + 1023) << 20, 0);
      int n = 0;
      for (int w = 0; w < 4; ++w)
        for (uint32_t m = S.klossy[jj][w]; m; m &= m - 1) {
          const int i = 32 * w + __ffs(m) - 1;
          if (n < LCAP) {
            const double k = (double)__uint_as_float((uint32_t)P.k[(base + j0 + jj) * D + i] << 16);
            S.kc_d[jj][n] = (float)(k - (double)read_fix_k(sK, jj, i) * pk);  // exact
            S.kc_i[jj][n] = (uint8_t)i;
          }
          ++n;
        }
      S.kc_n[jj] = (uint8_t)min(n, 255);
    }
    // ---------------- score MMAs: 7 groups x 64 columns (they run while the values are sliced) ----
    // Group g is issued by lane 0 of warp 2 g + 1: an issuing thread waits while the tensor core
    // takes its operands, so the groups' issuers share that wait (each commits to the barrier).
    if (lane == 0 && (warp & 1) && (warp >> 1) < NGS) {
      tc::fence_after_sync();
      const uint32_t aq = tc::smem_u32(sQ), bk = tc::smem_u32(sK);
      {
        const int g = warp >> 1;
        bool first = true;
        for (int s = 0; s < NQ; ++s) {
          const int t = g - s;
          if (t < 0 || t >= NK) continue;
          const uint32_t idesc = tc::idesc_i8(128, BN, s == NQ - 1, t == NK - 1);
          for (int ks = 0; ks < D / 32; ++ks) {
            uint64_t ad = tc::smem_desc(aq + s * Q_PLANE + ks * 2 * (BM / 8) * 128, (BM / 8) * 128, 128);
            uint64_t bd = tc::smem_desc(bk + t * K_PLANE + ks * 2 * KLBO, KLBO, 128);
            tc::mma_i8(tmem + BN * g, ad, bd, idesc, !first);
            first = false;
          }
        }
      }
      tc::mma_commit(tc::smem_u32(&S.bar));
    }

    // ---------------- V tile -> digit planes (thread: channel tid % 128, keys 16 (tid / 128) ..) ------
    // Against the block's channel exponent: through fp32 unless some value is NaN / inf or loses
    // bits below the window (then element by element, flagging its key).
    {
      const int c = tid & 127, vq = tid >> 7;
      const int ve = S.ve[c];
      const int lsb = ve == INT32_MIN ? 0 : ve - FV;
      const uint32_t thr = (uint32_t)max(lsb + 134, 0) << 7;  // nonzero |v| bits below this lose bits
      uint32_t b16[16];
      uint32_t flag = 0;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = 16 * vq + jj;
        b16[jj] = (j0 + j < maxlen) ? (uint32_t)P.v[(base + j0 + j) * DV + c] : 0u;
        const uint32_t u = b16[jj] & 0x7FFFu;
        flag |= (uint32_t)(u >= 0x7F80u) | (uint32_t)(u - 1u < thr - 1u);
      }
      uint32_t x[16];
      // (a channel without finite nonzero values has lsb 0: zeros convert exactly, NaN / inf go
      // to the flagged path)
      if (!flag && lsb >= -126) {
        const float sc = scale_of(lsb);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) x[jj] = fixf_lo(b16[jj], sc);
      } else {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j = 16 * vq + jj;
          int lost = 0, bad = 0;
          const int32_t f = fixq(b16[jj], lsb, lost, bad);
          if (bad) atomicOr(&S.kbad[j], 1);
          if (lost) atomicOr(&S.vlossy[j], 1);
          x[jj] = (uint32_t)f;
        }
      }
      uint4 pl[NV];
      planes16<NV>(x, pl);
#pragma unroll
      for (int p = 0; p < NV; ++p) *(uint4*)(sV + p * V_PLANE + tc::kmajor_off(c, 16 * vq, DV)) = pl[p];
    }
    tc::fence_async_smem();
    __syncthreads();
    EA_PT(1)

    if (tid < BN)
      S.kmeta[tid] = ((uint32_t)S.klsb[tid] & 0xFFFFu) |
                     ((S.klossy[tid][0] | S.klossy[tid][1] | S.klossy[tid][2] | S.klossy[tid][3]) ? 1u << 16 : 0u) |
                     (S.kbad[tid] ? 1u << 17 : 0u);
    {
      const bool okw = tc::mbar_wait(&S.bar, phase, P.wait_debug);
      phase ^= 1;
      // block-wide vote: a wait that gave up ends the tile loop for every thread together
      if (!__syncthreads_and(okw)) {
        ok_wait = false;
        break;
      }
    }
    tc::fence_after_sync();
    EA_PT(2)

    // ---------------- pass 1: certified logits of (r, keys 16 u4 ..) ----------------
    bool any_unc = false;
    {
      const int qlsb = S.qlsb[r];
      const bool qlossy = (S.qlossy[r][0] | S.qlossy[r][1] | S.qlossy[r][2] | S.qlossy[r][3]) != 0;
      const int nqc = S.qc_n[r];
      const bool qlist = nqc <= LCAP && qlsb >= -1000;  // the row's lost parts are all listed
      int rstat = ST_OK;
      // the tile bound of the certified logits: w = RN24(2^t) <= 2^(floor(t) + 1) < 2^(ceil(t) + 1),
      // and ceil is monotone (the ceiling of the largest logit); |t| >= 2^30 goes to tier 3
      float tmax = -INFINITY, tmin = INFINITY;
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t dg[NGS][4];
#pragma unroll
        for (int g = 0; g < NGS; ++g) tc::tmem_ld4(tlane + BN * g + 16 * u4 + 4 * c4, dg[g]);
        tc::tmem_wait_ld();
        EA_PT(13)
        // the binary64 fast path for the four keys (straight-line, interleaved), then the rare keys
        // it leaves to the integer evaluation: NaN/inf keys, lossy windows, results it cannot certify
        int64_t acc[4];
        uint32_t outv[4], slow = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int kj = 16 * u4 + 4 * c4 + u;
          const uint32_t km = S.kmeta[kj];
          const uint32_t lo4[4] = {dg[0][u], dg[1][u], dg[2][u], dg[3][u]};
          const uint32_t hi3[3] = {dg[4][u], dg[5][u], dg[6][u]};
          acc[u] = recomb<4>(lo4) + (int64_t)((uint64_t)recomb<3>(hi3) << 32);
          uint32_t fb;
          const bool ok = f64::logit_f64(acc[u], qlsb + (int32_t)(int16_t)(km & 0xFFFFu), am_d, P.ae, fb);
          const bool live = myrow >= 0 && j0 + kj < mylen;
          outv[u] = live ? fb : T_MASKED;
          if (live && (!ok || qlossy || (km >> 16) != 0)) slow |= 1u << u;
        }
        // a q row whose window lost bits, against keys that lost none: its exact correction
        // sum_e dq_e K_(key, i_e) 2^klsb for the four keys together (interleaved), from the row's list
        if (qlossy && qlist) {
          double cr[4] = {0.0, 0.0, 0.0, 0.0}, ca[4] = {0.0, 0.0, 0.0, 0.0};
          for (int e = 0; e < nqc; ++e) {
            const int i = S.qc_i[r][e];
            const double dq = (double)S.qc_d[r][e];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int kj = 16 * u4 + 4 * c4 + u;
              const int klsb = (int32_t)(int16_t)(S.kmeta[kj] & 0xFFFFu);
              const double t = dq * ((double)read_fix_k(sK, kj, i) * __hiloint2double((klsb + 1023) << 20, 0));
              cr[u] += t;  // dq K 2^klsb: exact products (at most 8 x 27 bits), one rounding per sum
              ca[u] += fabs(t);
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int kj = 16 * u4 + 4 * c4 + u;
            const uint32_t km = S.kmeta[kj];
            if (!((slow >> u) & 1u) || (km >> 16) != 0) continue;  // lossy keys: the general path
            uint32_t fb;
            const double cerr = (double)(nqc + 2) * 1.1102230246251565e-16 * ca[u] * 1.000001;
            const int sexp = qlsb + (int32_t)(int16_t)(km & 0xFFFFu);
            if (sexp - qlsb >= -1000 && f64::logit_f64_corr(acc[u], sexp, cr[u], cerr, am_d, P.ae, fb)) {
              outv[u] = fb;
              slow &= ~(1u << u);
            }
          }
        }
        EA_PT(14)
        for (uint32_t m = slow; m; m &= m - 1) {
          const int u = __ffs(m) - 1;
          const int kj = 16 * u4 + 4 * c4 + u;
          const uint32_t km = S.kmeta[kj];
          uint32_t out = T_MASKED;
          if ((km >> 17) & 1u) {
            rstat = ST_DOMAIN;
          } else {
            const bool klossy = ((km >> 16) & 1u) != 0;
            const int sexp = qlsb + (int32_t)(int16_t)(km & 0xFFFFu);
            uint32_t fb;
            bool done = false, differ = false;
            uint64_t err = 0;
            if (qlossy || klossy) {
              // first the exact correction of the lossy elements, then the truncation bound
              double cerr, corr;
              if (!score_corr_cached(S, sQ, sK, r, kj, qlsb, sexp - qlsb, corr, cerr))
                corr = score_corr(S, sQ, sK, r, kj, P.q + (int64_t)myrow * D, P.k + (base + j0 + kj) * D, qlsb,
                                  sexp - qlsb, cerr);
              done = sexp - qlsb >= -1000 && qlsb >= -1000 &&
                     f64::logit_f64_corr(acc[u], sexp, corr, cerr, am_d, P.ae, fb);
              if (!done) {
                err = score_err(S, sQ, sK, r, kj);
                done = f64::logit_interval_f64(acc[u], err, sexp, am_d, P.ae, fb, differ);
              }
            }
            if (done) {
              out = fb;
            } else if (differ) {
              out = T_UNCERT;
            } else {
              Rnd t = rnd_zero();
              const int ls = (qlossy || klossy) ? logit_bounded(acc[u], err, sexp, P.am, P.ae, t)
                                                : logit_exact_ool(acc[u], sexp, P.am, P.ae, t);
              if (ls == LOGIT_OK) out = rnd_to_f32_bits(t);
              else if (ls == LOGIT_UNCERTIFIED) out = T_UNCERT;
              else rstat = ST_DOMAIN;
            }
          }
          outv[u] = out;
        }
        EA_PT(15)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          sT[r * T_PITCH + 16 * u4 + 4 * c4 + u] = outv[u];
          const float tf = __uint_as_float(outv[u]);
          if (fabsf(tf) < 1073741824.0f) {  // false for the NaN markers
            tmax = fmaxf(tmax, tf);
            tmin = fminf(tmin, tf);
          } else if (outv[u] != T_MASKED && outv[u] != T_UNCERT) {
            rstat = max(rstat, (int)ST_TIER3);  // |t| >= 2^30: the wide tier (whose exponents hold it)
          }
          any_unc |= outv[u] == T_UNCERT;
        }
      }
      if (rstat != ST_OK) atomicMax(&S.rst[r], rstat);
      S.rt[u4][r] = tmax == -INFINITY ? INT32_MIN : __float2int_ru(tmax) + 1;
      tlo = fminf(tlo, tmin);
    }
    tc::fence_before_sync();
    const bool tile_unc = __syncthreads_or(any_unc);
    EA_PT(3)

    // ---------------- exact scores of the uncertified pairs, one warp per pair ----------------
    // entry e = warp + 16 (32 it + lane): a row with many uncertified pairs spreads over every warp.
    // Then the tile bounds again, over the exact logits too.
    if (tile_unc) {
      for (int it = 0; it < BM * BN / (32 * NWARPS); ++it) {
        const int e = warp + NWARPS * (32 * it + lane);
        uint32_t hit = __ballot_sync(0xffffffffu, sT[(e >> 6) * T_PITCH + (e & 63)] == T_UNCERT);
        while (hit) {
          const int src = __ffs(hit) - 1;
          hit &= hit - 1;
          const int ee = warp + NWARPS * (32 * it + src);
          const int pr = ee >> 6, pk = ee & 63;
          Rnd t = rnd_zero();
          const int ls = warp_exact_logit(P.q, P.k, P.am, P.ae, S.rows[pr], base + j0 + pk, t);
          if (lane == 0) {
            if (ls == LOGIT_OK) {
              sT[pr * T_PITCH + pk] = rnd_to_f32_bits(t);
            } else {
              sT[pr * T_PITCH + pk] = T_MASKED;
              atomicMax(&S.rst[pr], ST_DOMAIN);
            }
            ++n_exact;
          }
        }
      }
      __syncthreads();
      {
        float tmax = -INFINITY;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const uint32_t tb = sT[r * T_PITCH + 16 * u4 + u];
          const float tf = __uint_as_float(tb);
          if (fabsf(tf) < 1073741824.0f) {
            tmax = fmaxf(tmax, tf);
            tlo = fminf(tlo, tf);
          } else if (tb != T_MASKED && tb != T_UNCERT) {
            atomicMax(&S.rst[r], ST_TIER3);  // |t| >= 2^30: the wide tier
          }
        }
        S.rt[u4][r] = tmax == -INFINITY ? INT32_MIN : __float2int_ru(tmax) + 1;
      }
      __syncthreads();
    }
    EA_PT(4)

    // ---------------- pass 2: weights, W digits ----------------
    EA_PT(11)
    const int32_t Rt = max(max(S.rt[0][r], S.rt[1][r]), max(S.rt[2][r], S.rt[3][r]));
    {
      uint64_t wsum = 0, vwsum = 0;
      uint32_t nlw = 0;
      int rstat = ST_OK;
#pragma unroll 1
      for (int wd = 0; wd < 4; ++wd) {
        // the binary64 fast path for the four keys (straight-line, interleaved); the integer
        // evaluation for the rare ones it leaves (|t| >= 2^22, or too close to a midpoint)
        uint64_t Wv[4];
        uint32_t slow = 0, counted = 0;  // keys for the integer path; keys that enter the sums
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int kj = 16 * u4 + 4 * wd + u;
          const uint32_t tb = sT[r * T_PITCH + kj];
          const float tf = __uint_as_float(tb);
          uint32_t M;
          int32_t E;
          const bool ok = f64::weight_f64(tb, S.td, M, E);
          const bool live = tb != T_MASKED && Rt != INT32_MIN;
          // w < 2^(t + 1) <= 2^(Rt - 48): W = 0, a truncated (nonzero) weight
          const bool tiny = tf > -1073741824.0f && (double)tf < (double)Rt - 49.0;
          // W = floor(M 2^sh) with M < 2^24 and sh <= 24 (w < 2^Rt): a left shift fits in 48 bits,
          // a right shift stays in 32 (clamped to 31 below 2^-31, which the lost flag covers)
          const int sh = E + FW - Rt;
          const int rs = min(max(-sh, 0), 31);
          const uint32_t Wr = sh <= -32 ? 0u : M >> rs;
          const uint64_t W = sh >= 0 ? (uint64_t)M << min(sh, 24) : (uint64_t)Wr;
          const bool lost = sh < 0 && (sh <= -32 || (M & ((1u << rs) - 1u)) != 0u);
          Wv[u] = (live && !tiny && ok) ? W : 0ull;
          if (live && (tiny || (ok && lost))) ++nlw;
          if (live && !tiny && !ok) slow |= 1u << u;
          if (live && (tiny || ok)) counted |= 1u << u;
        }
        for (uint32_t m = slow; m; m &= m - 1) {
          const int u = __ffs(m) - 1;
          const Rnd t = rnd_from_f32(sT[r * T_PITCH + 16 * u4 + 4 * wd + u]);
          uint32_t M;
          int64_t E;
          int ws = weight_ool(t, M, E);
          if (ws == W_RISKY) {
            ++n_wide;
            ws = wide_weight(t, M, E);
          }
          uint64_t W = 0;
          if (ws != W_OK) {
            rstat = ST_TIER3;
          } else {
            counted |= 1u << u;
            const int sh = (int)(E + FW - Rt);
            if (sh >= 0) {
              W = (uint64_t)M << sh;
            } else if (sh > -64) {
              W = (uint64_t)M >> (-sh);
              nlw += (W << (-sh)) != M;
            } else {
              ++nlw;
            }
          }
          Wv[u] = W;
        }
        uint32_t wlo[4], whi[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if ((counted >> u) & 1u) {
            wsum += Wv[u];
            if (S.vlossy[16 * u4 + 4 * wd + u]) vwsum += Wv[u] + 1;
          }
          wlo[u] = (uint32_t)Wv[u];
          whi[u] = (uint32_t)(Wv[u] >> 32);
        }
        uint8_t* dst = sW + tc::kmajor_off(r, 16 * u4 + 4 * wd, BM);
        *(uint32_t*)(dst + 0 * W_PLANE) = pack4<0>(wlo[0], wlo[1], wlo[2], wlo[3]);
        *(uint32_t*)(dst + 1 * W_PLANE) = pack4<1>(wlo[0], wlo[1], wlo[2], wlo[3]);
        *(uint32_t*)(dst + 2 * W_PLANE) = pack4<2>(wlo[0], wlo[1], wlo[2], wlo[3]);
        *(uint32_t*)(dst + 3 * W_PLANE) = pack4<3>(wlo[0], wlo[1], wlo[2], wlo[3]);
        *(uint32_t*)(dst + 4 * W_PLANE) = pack4<0>(whi[0], whi[1], whi[2], whi[3]);
        *(uint32_t*)(dst + 5 * W_PLANE) = pack4<1>(whi[0], whi[1], whi[2], whi[3]);
      }
      EA_PT(12)
      S.zs[u4][r] = wsum;
      S.zl[u4][r] = nlw;
      S.vw[u4][r] = vwsum;
      if (rstat != ST_OK) atomicMax(&S.rst[r], rstat);
    }
    tc::fence_async_smem();
    __syncthreads();
    EA_PT(5)

    // ---------------- P.V MMAs in four rounds of two groups, drained into N ----------------
    // Round rd (groups 2 rd, 2 rd + 1) accumulates in TMEM columns 256 (rd % 2) ..; round rd + 1 is
    // issued before round rd is drained, so the tensor cores work while the CUDA cores drain, and
    // rounds 0 and 1 go out before the merge below, which they overlap. A round's commit goes to
    // the barrier of its parity (each completes once before it is waited on).
    // group 2 rd + i is issued by lane 0 of warp 4 rd + 2 i (as the score groups)
    auto issue_pv = [&](int rd) {
      if (lane != 0 || (warp >> 2) != rd || (warp & 1)) return;
      tc::fence_after_sync();
      const uint32_t aw = tc::smem_u32(sW), bv = tc::smem_u32(sV);
      {
        const int g = 2 * rd + ((warp >> 1) & 1);
        bool first = true;
        for (int s = 0; s < NW; ++s) {
          const int t = g - s;
          if (t < 0 || t >= NV) continue;
          const uint32_t idesc = tc::idesc_i8(128, DV, false, t == NV - 1);
          for (int ks = 0; ks < BN / 32; ++ks) {
            uint64_t ad = tc::smem_desc(aw + s * W_PLANE + ks * 2 * (BM / 8) * 128, (BM / 8) * 128, 128);
            uint64_t bd = tc::smem_desc(bv + t * V_PLANE + ks * 2 * (DV / 8) * 128, (DV / 8) * 128, 128);
            tc::mma_i8(tmem + 256 * (rd & 1) + DV * (g - 2 * rd), ad, bd, idesc, !first);
            first = false;
          }
        }
      }
      tc::mma_commit(tc::smem_u32(&S.bar_pv[rd & 1]));
    };
    issue_pv(0);
    issue_pv(1);
    pv_pending = 3;  // bit b: the barrier of parity b has a commit in flight
    // ---------------- merge Z, rescale N, bounds ----------------
    int sh_base = 0;  // (Rt - FW - FV) - (R - FN): shift of a W.Vfix unit into N units
    if (Rt != INT32_MIN) {
      const int32_t Rn = R == R_EMPTY ? Rt : max(R, Rt);
      if (R != R_EMPTY && Rn > R) {
        const int d = Rn - R, dc = min(d, 63);  // d > 0: an arithmetic right shift is the floor
#pragma unroll
        for (int c = 0; c < 32; ++c) N[c] >>= dc;
        Nerr = scale_ceil(Nerr, -d) + 1;
        int lost;
        Z = floor_shift(Z, -d, lost);
        Zerr = scale_ceil(Zerr, -d) + (uint64_t)lost;
      }
      R = Rn;
      const uint64_t zt = S.zs[0][r] + S.zs[1][r] + S.zs[2][r] + S.zs[3][r];
      const uint64_t nlw = (uint64_t)S.zl[0][r] + S.zl[1][r] + S.zl[2][r] + S.zl[3][r];
      const uint64_t vw = S.vw[0][r] + S.vw[1][r] + S.vw[2][r] + S.vw[3][r];
      const int zsh = (Rt - FW) - (R - FZ);  // Z units
      int lost = 0;
      Z += floor_shift((int64_t)zt, zsh, lost);
      Zerr += scale_ceil(nlw, zsh) + (uint64_t)lost;
      sh_base = (Rt - FW - FV) - (R - FN);
      // truncated weights: < 1 W unit times |v| < 2^VE -> 2^(Rt - FW - R + FN) N units each
      Nerr += scale_ceil(nlw, sh_base + FV);
      // truncated values (keys flagged lossy): < W + 1 W units times one V unit
      Nerr += scale_ceil(vw, sh_base);
      // floors of the per-round shifts (rounds start at groups 0, 2, 4, 6)
#pragma unroll
      for (int g = 0; g < NGP; g += 2) Nerr += (8 * g + sh_base < 0) ? 1 : 0;
    }

    EA_PT(6)
#pragma unroll 1
    for (int rd = 0; rd < 4; ++rd) {
      {
        const bool okw = tc::mbar_wait(&S.bar_pv[rd & 1], (pv_phase >> (rd & 1)) & 1u, P.wait_debug);
        pv_phase ^= 1u << (rd & 1);
        pv_pending &= ~(1u << (rd & 1));
        if (!__syncthreads_and(okw)) {
          ok_wait = false;
          break;
        }
      }
      tc::fence_after_sync();
      EA_PT(7)
      {  // warp-collective loads: every lane takes part (rows without visible keys add zeros)
        // floor(X 2^s) as (X << l) >> r: s <= 38 and the round's |X| < 2^33 (so X 2^l < 2^63), and
        // a right shift clamped to 63 still floors
        const int s = 16 * rd + sh_base;
        const int l = max(s, 0), rr = min(max(-s, 0), 63);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint32_t dg[2][8];
          tc::tmem_ld8(tlane + 256 * (rd & 1) + 32 * u4 + 8 * c8, dg[0]);
          tc::tmem_ld8(tlane + 256 * (rd & 1) + DV + 32 * u4 + 8 * c8, dg[1]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t d2[2] = {dg[0][u], dg[1][u]};
            N[8 * c8 + u] += (int64_t)((uint64_t)recomb<2>(d2) << l) >> rr;
          }
        }
      }
      tc::fence_before_sync();
      __syncthreads();
      EA_PT(8)
      if (rd + 2 < 4) {
        issue_pv(rd + 2);
        pv_pending |= 1u << (rd & 1);
      }
    }
    if (!ok_wait) break;  // uniform: set by the block vote
  }
  if (!ok_wait) {
    // a wait that gave up: the MMAs still in flight get a bounded wait before TMEM is released
    tc::mbar_wait(&S.bar, phase ^ 1u, P.wait_debug);
    for (int b = 0; b < 2; ++b)
      if ((pv_pending >> b) & 1u) tc::mbar_wait(&S.bar_pv[b], (pv_phase >> b) & 1u, P.wait_debug);
  }

  EA_PT(9)
  // the row's logits spanning more than SPREAD_CHECK below its bound: tier 3 decides the
  // reference's exponent-spread rule (the four threads of a row pool their lowest logits)
  S.rt[u4][r] = tlo == INFINITY ? INT32_MAX : __float2int_rd(tlo);
  __syncthreads();
  if (u4 == 0 && R != R_EMPTY) {
    const int32_t lo = min(min(S.rt[0][r], S.rt[1][r]), min(S.rt[2][r], S.rt[3][r]));
    if (lo != INT32_MAX && (int64_t)R - lo > SPREAD_CHECK) atomicMax(&S.rst[r], ST_TIER3);
  }
  __syncthreads();
  // ---------------- export (KV-sharded runs) or finalise ----------------
  // KV splits (gridDim.y > 1) write split partials, merged exactly by the split combine; a
  // KV-sharded run exports its partials in the same one-sided form
  const bool exporting = P.export_partials || gridDim.y > 1;
  const int64_t so = (int64_t)blockIdx.y * P.rows;
  int32_t* xR = gridDim.y > 1 ? P.pR + so : P.xR;
  int64_t* xZ = gridDim.y > 1 ? P.pZ + so : P.xZ;
  uint64_t* xZe = gridDim.y > 1 ? P.pZe + so : P.xZe;
  int32_t* xSt = gridDim.y > 1 ? P.pSt + so : P.xSt;
  int32_t* xNR = gridDim.y > 1 ? P.pNR + so * DV : P.xNR;
  int64_t* xN = gridDim.y > 1 ? P.pN + so * DV : P.xN;
  uint64_t* xNe = gridDim.y > 1 ? P.pNe + so * DV : P.xNe;
  if (exporting) {
    // partials in the one-sided form [N, N + Nerr] of ea_partials_t: this kernel's N interval is
    // [N - Nerr, N + Nerr], in units 2^(R + VE_c - FN) = 2^(NR - FZ) with NR = R + VE_c
    if (myrow >= 0) {
      const int st = ok_wait ? S.rst[r] : ST_TIER3;
      if (u4 == 0) {
        xR[myrow] = R;
        xZ[myrow] = Z;
        xZe[myrow] = Zerr;
        xSt[myrow] = st;
      }
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int ch = 32 * u4 + c, ve = S.ve[ch];
        const int64_t o = (int64_t)myrow * DV + ch;
        const bool empty = R == R_EMPTY || ve == INT32_MIN;
        xNR[o] = empty ? R_EMPTY : R + ve;
        xN[o] = empty ? 0 : N[c] - (int64_t)Nerr;
        xNe[o] = empty ? 0 : 2 * Nerr;
      }
    }
  } else {
    const int st = S.rst[r];
    const int prec = P.fp32 ? FP32_P : BF16_P, qmin = P.fp32 ? FP32_QMIN : BF16_QMIN;
    uint32_t outw[16];  // bf16 results, two per word (fp32 results are recomputed when stored)
    bool ok = ok_wait && st == ST_OK;
    // one pair of divisor reciprocals for the row's channels
    const double rzl = f64::recip_f64(Z), rzh = f64::recip_f64(Z + (int64_t)Zerr);
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      Rnd x = rnd_zero();
      const int ve = S.ve[32 * u4 + c];
      if (ok && R != R_EMPTY && ve != INT32_MIN) {
        // binary64 first; the integer division decides what it cannot certify
        const int64_t nl = N[c] - (int64_t)Nerr, nh = N[c] + (int64_t)Nerr;
        const int64_t nu = (int64_t)R + ve - FN, zu = (int64_t)R - FZ;
        const int cf = f64::certify_ratio_f64_rcp(nl, nh, nu, Z, Z + (int64_t)Zerr, rzl, rzh, zu, prec, qmin, 127, x);
        if (cf == 0) ok = false;
        else if (cf < 0) ok &= certify_ratio_lh(nl, nh, nu, Z, Z + (int64_t)Zerr, zu, prec, qmin, 127, x);
      }
      const uint32_t b = rnd_to_bf16_bits(x);
      if (c & 1) outw[c >> 1] |= b << 16;
      else outw[c >> 1] = b;
    }
    if (!ok) atomicAnd(&S.rok[r], 0);
    __syncthreads();
    if (myrow >= 0) {
      const bool rowok = S.rok[r] != 0;
      if (st == ST_DOMAIN) {
        if (P.fp32) {
          uint4* o = (uint4*)((uint32_t*)P.out + (int64_t)myrow * DV + 32 * u4);
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8) o[q8] = make_uint4(0, 0, 0, 0);
        } else {
          uint4* o = (uint4*)((uint16_t*)P.out + (int64_t)myrow * DV + 32 * u4);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) o[q4] = make_uint4(0, 0, 0, 0);
        }
        if (u4 == 0) {
          P.flags[myrow] = 2;
          stat_add(P, STAT_DOMAIN_ROWS, 1);
        }
      } else if (!rowok || forced_uncertified(P, myrow)) {
        if (u4 == 0) leave_tier(P, myrow, rowok);
      } else if (P.fp32) {
        // every channel certified: round again, now keeping the fp32 results (4 per store)
        uint32_t* o = (uint32_t*)P.out + (int64_t)myrow * DV + 32 * u4;
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          uint32_t f[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = 4 * c4 + u;
            Rnd x = rnd_zero();
            const int ve = S.ve[32 * u4 + c];
            if (R != R_EMPTY && ve != INT32_MIN) {
              const int64_t nl = N[c] - (int64_t)Nerr, nh = N[c] + (int64_t)Nerr;
              const int64_t nu = (int64_t)R + ve - FN, zu = (int64_t)R - FZ;
              if (f64::certify_ratio_f64_rcp(nl, nh, nu, Z, Z + (int64_t)Zerr, rzl, rzh, zu, FP32_P, FP32_QMIN, 127,
                                             x) < 0)
                certify_ratio_lh(nl, nh, nu, Z, Z + (int64_t)Zerr, zu, FP32_P, FP32_QMIN, 127, x);
            }
            f[u] = rnd_to_f32_bits(x);
          }
          *(uint4*)(o + 4 * c4) = make_uint4(f[0], f[1], f[2], f[3]);
        }
        if (u4 == 0) P.flags[myrow] = 0;
      } else {
        uint4* o = (uint4*)((uint16_t*)P.out + (int64_t)myrow * DV + 32 * u4);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) o[q4] = make_uint4(outw[4 * q4], outw[4 * q4 + 1], outw[4 * q4 + 2], outw[4 * q4 + 3]);
        if (u4 == 0) P.flags[myrow] = 0;
      }
    }
  }
  n_exact = __reduce_add_sync(0xffffffffu, n_exact);
  n_wide = __reduce_add_sync(0xffffffffu, n_wide);
  if (lane == 0) {
    stat_add(P, STAT_SCORE_EXACT, n_exact);
    stat_add(P, STAT_WEIGHT_WIDE, n_wide);
  }
  if (tid == 0) {
    unsigned long long pairs = 0;
    for (int i = 0; i < BM; ++i) pairs += (unsigned long long)S.len[i];
    stat_add(P, STAT_PAIRS, pairs);
    stat_add(P, STAT_TC_PAIRS, pairs);
    if (!ok_wait) stat_add(P, STAT_WAIT_EXPIRED, 1);  // a bounded wait gave up
  }
  EA_PT(10)
  EA_PT_FLUSH
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_free(tmem, TMEM_COLS);
}

}  // namespace tck

cudaError_t launch_tc_prefill(const Prob& P, const int32_t* block_rows, int64_t nblocks, cudaStream_t st) {
  // the shared-memory opt-in is a property of the function on a device: set it once per device
  // (not per launch, so a launch inside a stream capture issues nothing but the kernel)
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tck::tc_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)tck::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  // KV splits on grid.y (the split partials are merged by the split combine)
  dim3 grid((unsigned)nblocks, (unsigned)(P.splits > 1 ? P.splits : 1));
  tck::tc_prefill_kernel<<<grid, tck::THREADS, tck::SMEM_BYTES, st>>>(P, block_rows);
  return cudaGetLastError();
}

size_t tc_prefill_smem_bytes() { return tck::SMEM_BYTES; }

}  // namespace ea

#ifdef EA_PHASE_TIMERS
// phase clocks of the tensor-core kernel (timer builds only): copies and clears the 16 counters
extern "C" int ea_debug_phase_cycles(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, ea::tck::g_phase_cycles, sizeof(unsigned long long) * 16);
  unsigned long long z[16] = {0};
  return cudaMemcpyToSymbol(ea::tck::g_phase_cycles, z, sizeof(z)) == cudaSuccess ? 0 : -4;
}
#endif

namespace ea {

}  // namespace ea
