// Tensor-core (tcgen05 / TMEM) tier-1 kernel of certified ExactAttention for decode: a few query
// rows (one GQA group of one sequence, at most 8) against a long key sequence, d = dv = 128.
//
// The prefill kernel puts 128 query rows on the MMA's M side; a decode group has 1-8 rows, so
// here the KEYS take the M side and the rows' digits go to N:
//   scores   S^T[key, (g, s)] = K_t . Q_s for key digit planes t (A, 128 keys x 128 dims) against
//            one B tile holding every row's 4 query digit planes (N = 32 = 8 rows x 4 digits).
//            Query digits are balanced (signed bytes) so one B tile has one signedness.
//   P.V      O^T[c, (g, w)] = V_u . W_w for value digit planes u (A, 128 channels x 128 keys)
//            against one B tile of every row's 6 weight digit planes (N = 48); values in a 31-bit
//            window against the channel's running maximum, 4 digits.
// Digit products are grouped by digit position on the CUDA cores (int32 sums) and recombined
// exactly in int64, with the same fixed-point windows, bounds and certification as the prefill
// kernel. Each CTA takes one (segment, split): the split's 128-key tiles arrive by bulk copies
// (cp.async.bulk, completing on an mbarrier) into a raw staging buffer one tile ahead of the
// slicing. Every CTA writes its rows' split partials; the split combine merges them (any split
// count gives the same bits) and sends uncertified rows to tier 3.
//
// Thread roles (512 threads, warp-specialised): warps 8-15 (producers) turn the raw tiles into
// digit planes, issue the score MMAs and the next tiles' bulk copies; warps 0-7 (consumers, the
// TMEM lane quadrant = warp % 4) compute logits, weights and W digits, issue the P.V MMAs, and keep
// the running sums (pass 1 / pass 2: lane = key; drain: lane = channel; rows g = warp / 4 + 2 i).
// The slicing of tile i + 1 overlaps the epilogue of tile i; mbarriers carry the hand-offs (raw
// K / V landed, score MMAs done, pass 1 done, value digits ready, P.V done) and every wait is
// bounded.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ea_core.cuh"
#include "ea_fast64.cuh"
#include "ea_numerics.h"
#include "ea_tables.cuh"
#include "ea_tc_common.cuh"
#include "ea_tcgen05.cuh"

namespace ea {
namespace tcd {

using namespace tcc;

#ifdef EA_PHASE_TIMERS
__device__ unsigned long long g_phase_cycles[16];
#endif

constexpr int BK = 128, D = 128, DV = 128, GD = 8;
constexpr int NQ = 4, NK = 4, NW = 6, NV = 4;
constexpr int FW = 48, FV = 31;  // V: 31-bit window, 4 digits (few values fall below it)
constexpr int THREADS = 512, NWARPS = THREADS / 32;
constexpr int NWGC = 2;         // consumer warpgroups (warps 0-7); warps 8-15 are the producers
constexpr int RPT_MAX = GD / NWGC;  // row slots per consumer thread for a full segment of GD rows
constexpr uint32_t VLCAP = 4;
constexpr uint32_t VL_BOUNDED = 1u << 20;  // marks a channel without digits (all values bounded)
constexpr uint32_t TMEM_COLS = 512;
constexpr int NSQ = NQ * GD;  // score B rows: n = 4 g + s
constexpr int NSW = NW * GD;  // P.V B rows: n = 6 g + w
constexpr uint32_t COL_O = 128;  // P.V accumulators: COL_O + 48 u + n (scores: 32 t + n)

constexpr uint32_t RAW_K = BK * D * 2;  // 32768
constexpr uint32_t K_PLANE = BK * D;    // 16384
constexpr uint32_t V_PLANE = DV * BK;   // 16384
constexpr uint32_t OFF_RAWK = 0;
constexpr uint32_t OFF_RAWV = OFF_RAWK + RAW_K;
constexpr uint32_t OFF_K = OFF_RAWV + RAW_K;
constexpr uint32_t OFF_V = OFF_K + NK * K_PLANE;
constexpr uint32_t OFF_Q = OFF_V + NV * V_PLANE;
constexpr uint32_t OFF_W = OFF_Q + NSQ * D;
constexpr uint32_t OFF_T = OFF_W + NSW * BK;
constexpr uint32_t OFF_SMALL = OFF_T + GD * BK * 4;

struct Small {
  uint32_t klossy[BK][4];
  int32_t klsb[BK];
  int32_t kbad[BK];
  // value metadata of the last two tiles (by tile parity): the producers write tile i + 1's while
  // the consumers still read tile i's
  uint32_t vlmask[2][DV][4];  // keys whose value in channel c lost bits in the V window
  // per channel, up to VLCAP values that lost bits in the V window, with their lost parts (units
  // 2^(lsb_c - 24)), added back exactly in the drain: (key | still-lossy << 8), part
  uint32_t vl_n[2][DV];
  uint16_t vl_k[2][DV][4];
  int32_t vl_dx[2][DV][4];
  int32_t ve[2][DV];   // running channel exponent VE_c (|v| < 2^VE_c so far), by tile parity
  int16_t ve4[4][DV];  // per key quarter maxima of the current tile (INT16_MIN: none)
  uint64_t td[256];  // binary64 2^(j/256) of the fast weight path
  int32_t rows[GD];
  int32_t len[GD];
  int32_t qlsb[GD];
  int32_t rst[GD];
  uint32_t qlossy[GD][4];
  int32_t rt[4][GD];    // per lane quadrant
  int32_t rtlo[4][GD];  // lowest floor(t) per lane quadrant (the exponent-spread check)
  uint64_t zs[4][GD];
  uint32_t zl[4][GD];
  // producer -> consumer: raw K / V tiles landed (bulk copies), score MMAs done, value digits
  // ready; consumer -> producer: pass 1 done, P.V MMAs done
  uint64_t bar_rk, bar_rv, bar_smma, bar_vready, bar_p1, bar_pv;
  int32_t abort;  // a bounded wait gave up in either role
  uint32_t tmem;
  int32_t nrows;
  int32_t maxlen;
  int32_t row0;
};

constexpr uint32_t SMEM_BYTES = OFF_SMALL + sizeof(Small);
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(OFF_K % 1024 == 0 && OFF_Q % 16 == 0 && OFF_W % 16 == 0, "operand alignment");

// first K/V row and the number of contiguous rows from the segment's key j on (RANGE: the rest
// of the range; PAGED: the rest of the page)
__device__ __forceinline__ int64_t run_start(const Prob& P, int32_t row0, int64_t j, int64_t& run) {
  if (P.kind == MASK_RANGE) {
    run = INT64_MAX;
    return P.kv_base[row0] + j;
  }
  const int64_t b = row0 / P.hq;
  const int kvh = (int)(row0 - b * P.hq) / P.group;
  const int64_t page = P.page_table[b * P.max_pages + j / P.page_size];
  run = P.page_size - j % P.page_size;
  return (page * P.hkv + kvh) * P.page_size + (j % P.page_size);
}

// One warp: bulk copies of keys [j0, j0 + n) of `src` (K or V, 128 bf16 per row) into the raw
// tile `raw`; lane 0 arms the barrier. RANGE: one contiguous run from `kvbase` (the segment's
// kv_base, read once per CTA). PAGED: one run per page touched, run r issued by lane r % 32, each
// lane reading its own page-table entry (or taking it from page_pref, read a tile ahead), so the
// lookups overlap instead of chaining.
__device__ __forceinline__ void fetch_rows(const Prob& P, const uint16_t* src, int32_t row0, int64_t kvbase, int64_t j0, int n,
                           uint8_t* raw, uint64_t* bar, int64_t page_pref = -1) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) tc::mbar_arrive_expect_tx(bar, (uint32_t)n * D * 2u);
  __syncwarp();
  if (P.kind == MASK_RANGE) {
    if (lane == 0) tc::bulk_g2s(raw, src + (kvbase + j0) * D, (uint32_t)n * D * 2, bar);
    return;
  }
  const int ps = P.page_size;
  const int64_t b = row0 / P.hq;
  const int kvh = (int)(row0 - b * P.hq) / P.group;
  const int64_t p0 = j0 / ps, p1 = (j0 + n - 1) / ps;  // pages touched
  for (int64_t pg = p0 + lane; pg <= p1; pg += 32) {
    const int64_t ks = pg == p0 ? j0 : pg * ps;              // first key of the run
    const int64_t ke = min((pg + 1) * (int64_t)ps, j0 + n);  // one past its last key
    const int64_t page = (pg == p0 + lane && page_pref >= 0) ? page_pref : P.page_table[b * P.max_pages + pg];
    const int64_t kr = (page * P.hkv + kvh) * ps + (ks - pg * ps);
    tc::bulk_g2s(raw + (ks - j0) * (D * 2), src + kr * D, (uint32_t)(ke - ks) * D * 2, bar);
  }
}

// the page-table entry of lane's first page of the tile at j0 (PAGED; -1 otherwise)
__device__ __forceinline__ int64_t page_ahead(const Prob& P, int32_t row0, int64_t j0, int64_t kend) {
  if (P.kind != MASK_PAGED || j0 >= kend) return -1;
  const int lane = threadIdx.x & 31;
  const int64_t pg = j0 / P.page_size + lane;
  const int64_t plast = (min(j0 + BK, kend) - 1) / P.page_size;
  return pg <= plast ? (int64_t)P.page_table[(int64_t)(row0 / P.hq) * P.max_pages + pg] : -1;
}

// Named barrier over one warpgroup pair (256 threads) with an AND vote.
__device__ __forceinline__ bool group_sync_and(int id, bool p) {
  int r;
  asm volatile(
      "{\n\t.reg .pred q, rr;\n\t"
      "setp.ne.s32 q, %1, 0;\n\t"
      "bar.red.and.pred rr, %2, 256, q;\n\t"
      "selp.s32 %0, 1, 0, rr;\n\t}\n"
      : "=r"(r)
      : "r"((int)p), "r"(id)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool group_sync_or(int id, bool p) {
  int r;
  asm volatile(
      "{\n\t.reg .pred q, rr;\n\t"
      "setp.ne.s32 q, %1, 0;\n\t"
      "bar.red.or.pred rr, %2, 256, q;\n\t"
      "selp.s32 %0, 1, 0, rr;\n\t}\n"
      : "=r"(r)
      : "r"((int)p), "r"(id)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void group_sync(int id) { asm volatile("bar.sync %0, 256;" ::"r"(id) : "memory"); }

// an mbarrier arrival by one thread
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

// floor(x * 2^s) of an int128 (callers keep left shifts in range)
__device__ __forceinline__ i128 shift_floor128(i128 x, int s) {
  if (s >= 0) return (i128)((u128)x << s);
  return s <= -127 ? (x < 0 ? -1 : 0) : (x >> (-s));
}
// ceil(u * 2^s) as a u128 (s < 64)
__device__ __forceinline__ u128 scale_ceil128(u128 u, int s) {
  if (s >= 0) return u << s;
  const int r = -s;
  if (r >= 128) return u != 0;
  return (u >> r) + ((u & (((u128)1 << r) - 1)) != 0);
}

// The part of bf16 `bits` that truncation toward zero to a multiple of 2^lsb dropped, in units
// 2^(lsb - 24), itself truncated toward zero (< 2^24); `lost2` when bits remain below that unit.
__device__ __forceinline__ int32_t lost_part24(uint32_t bits, int lsb, int& lost2) {
  int32_t m, e;
  decode_bf16(bits, m, e);
  lost2 = 0;
  const uint32_t mag = (uint32_t)(m < 0 ? -m : m);
  const int s = lsb - e;  // the kept part is mag >> s
  if (s <= 0) return 0;
  const uint32_t low = s >= 31 ? mag : (mag & ((1u << s) - 1));  // units 2^e, < 2^9
  uint32_t dx;
  if (s <= 24) {
    dx = low << (24 - s);
  } else {
    const int r = s - 24;
    dx = r >= 32 ? 0u : (low >> r);
    lost2 = r >= 32 ? (low != 0) : ((dx << r) != low);
  }
  return m < 0 ? -(int32_t)dx : (int32_t)dx;
}

// q row g's fixed-point element i from its balanced digit planes in the score B tile
__device__ __forceinline__ int32_t q_fix(const uint8_t* sQ, int g, int i) {
  int32_t x = 0;
#pragma unroll
  for (int t = NQ - 1; t >= 0; --t) x = x * 256 + (int32_t)(int8_t)sQ[tc::kmajor_off(4 * g + t, i, NSQ)];
  return x;
}

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// RPT: row slots per consumer thread (rows h, h + NWGC, ..): segments of at most NWGC RPT rows.
// A smaller RPT keeps fewer running sums in registers (GQA groups of 2 need one slot).
template <int RPT>
__global__ void __launch_bounds__(THREADS, 1) tc_decode_kernel(Prob P, const int32_t* __restrict__ seg_rows) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* rawk = smem + OFF_RAWK;
  uint8_t* rawv = smem + OFF_RAWV;
  uint8_t* sK = smem + OFF_K;
  uint8_t* sV = smem + OFF_V;
  uint8_t* sQ = smem + OFF_Q;
  uint8_t* sW = smem + OFF_W;
  uint32_t* sT = (uint32_t*)(smem + OFF_T);
  Small& S = *(Small*)(smem + OFF_SMALL);
  EA_PT_DECL

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seg = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;

  // ---------------- segment rows and this split's key range ----------------
  if (tid < GD) {
    int32_t row;
    if (seg_rows) {
      row = seg_rows[(int64_t)seg * GD + tid];
    } else {  // PAGED: sequence seg / kv_heads, kv head seg % kv_heads, the group's q heads
      const int b = seg / P.hkv, kvh = seg % P.hkv;
      row = tid < P.group ? b * P.hq + kvh * P.group + tid : -1;
    }
    S.rows[tid] = row;
    S.len[tid] = row >= 0 ? (int32_t)row_len(P, row) : 0;
    S.rst[tid] = ST_OK;
  }
  for (int i = tid; i < DV; i += THREADS) S.ve[0][i] = S.ve[1][i] = INT32_MIN;
  for (int i = tid; i < GD * BK; i += THREADS) sT[i] = T_MASKED;
  if (tid < 256) S.td[tid] = f64::g_exp2_d64[tid];
  if (tid == 0) {
    tc::mbar_init(&S.bar_rk, 1);
    tc::mbar_init(&S.bar_rv, 1);
    tc::mbar_init(&S.bar_smma, NK);  // one commit per key digit's issuer
    tc::mbar_init(&S.bar_pv, NV);    // one commit per value digit's issuer
    tc::mbar_init(&S.bar_p1, 1);
    tc::mbar_init(&S.bar_vready, 1);
    S.abort = 0;
  }
  __syncthreads();
  if (tid == 0) {
    int n = 0, m = 0, first = -1;
    for (int g = 0; g < GD; ++g)
      if (S.rows[g] >= 0) {
        n = g + 1;
        m = max(m, S.len[g]);
        if (first < 0) first = S.rows[g];
      }
    S.nrows = n;
    S.maxlen = m;
    S.row0 = first;
  }
  __syncthreads();
  const int nrows = S.nrows;
  if (nrows == 0) return;  // uniform: an all-padding segment
  if (nrows > NWGC * RPT) {
    // more rows than this instantiation keeps sums for (a launch error): every row of the segment
    // goes to the exact tier, and the run is flagged
    for (int i = tid; i < nrows * (DV + 1); i += THREADS) {
      const int g = i / (DV + 1), ch = i % (DV + 1);
      const int32_t row = S.rows[g];
      if (row < 0) continue;
      const int64_t pi = (int64_t)split * P.rows + row;
      if (ch == DV) {
        P.pR[pi] = R_EMPTY;
        P.pZ[pi] = 0;
        P.pZe[pi] = 0;
        P.pSt[pi] = ST_TIER3;
      } else {
        P.pNR[pi * DV + ch] = R_EMPTY;
        P.pN[pi * DV + ch] = 0;
        P.pNe[pi * DV + ch] = 0;
      }
    }
    if (tid == 0) stat_add(P, STAT_UNRESOLVED, 1000000);
    return;
  }
  const int32_t row0 = S.row0;  // the segment's rows share their keys: address them through this one
  const int64_t maxlen = S.maxlen;
  const int64_t kbeg = maxlen * split / nsplit, kend = maxlen * (split + 1) / nsplit;
  const int ntiles = (int)((kend - kbeg + BK - 1) / BK);
  const int64_t kvbase = P.kind == MASK_RANGE ? P.kv_base[row0] : 0;
  if (warp == 0) tc::tmem_alloc(&S.tmem, TMEM_COLS);
  // the first tile's K (warp 15) and V (warp 14) fetches
  if (warp == NWARPS - 1 && ntiles > 0)
    fetch_rows(P, P.k, row0, kvbase, kbeg, (int)min((int64_t)BK, kend - kbeg), rawk, &S.bar_rk);
  if (warp == NWARPS - 2 && ntiles > 0)
    fetch_rows(P, P.v, row0, kvbase, kbeg, (int)min((int64_t)BK, kend - kbeg), rawv, &S.bar_rv);

  // ---------------- query rows -> balanced digit planes (warp g: row g) ----------------
  if (warp < GD) {
    const int g = warp;
    const int32_t row = S.rows[g];
    uint32_t bits[4];
    int lead = INT32_MIN, bad = 0;
#pragma unroll
    for (int m4 = 0; m4 < 4; ++m4) {
      bits[m4] = row >= 0 ? (uint32_t)P.q[(int64_t)row * D + lane + 32 * m4] : 0u;
      int32_t m, e;
      if (!decode_bf16(bits[m4], m, e)) bad = 1;
      if (m) lead = max(lead, lead_of(m, e));
    }
    lead = __reduce_max_sync(0xffffffffu, lead);
    bad = __reduce_or_sync(0xffffffffu, bad);
    const int lsb = lead == INT32_MIN ? 0 : lead + 1 - P.W;
#pragma unroll
    for (int m4 = 0; m4 < 4; ++m4) {
      const int i = lane + 32 * m4;
      int lost = 0, b2 = 0;
      const int32_t x = (bad || lead == INT32_MIN) ? 0 : fixq(bits[m4], lsb, lost, b2);
      const uint32_t lm = __ballot_sync(0xffffffffu, lost != 0);
      if (lane == 0) S.qlossy[g][m4] = lm;
      // balanced base-256 digits: x = sum_s d_s 256^s, d_s in [-128, 127] (|x| < 2^28)
      int32_t y = x;
#pragma unroll
      for (int s = 0; s < NQ; ++s) {
        const int32_t dg = s == NQ - 1 ? y : (int32_t)(int8_t)(y & 0xFF);
        sQ[tc::kmajor_off(4 * g + s, i, NSQ)] = (uint8_t)(int8_t)dg;
        y = (y - dg) >> 8;
      }
    }
    if (lane == 0) {
      S.qlsb[g] = lsb;
      if (bad && row >= 0) S.rst[g] = ST_DOMAIN;
    }
  }
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = S.tmem;
  unsigned n_exact = 0, n_wide = 0;
  bool ok_wait = true;
  const double am_d = (double)P.am;
  // consumer state (rows h, h + NWGC, .. of channel c), live until the partials are written
  const int h = warp >> 2, c = 32 * (warp & 3) + lane;
  // Fraction bits of this CTA's Z and N windows: the headroom only has to cover the split's own
  // keys (61 - ceil(log2 keys)), which keeps more bits than the row-wide P.FZ; the windows are
  // converted to P.FZ units (interval ends rounded outwards) when the partials are written.
  int klog = 1;
  while (klog < 62 && ((int64_t)1 << klog) < kend - kbeg) ++klog;
  const int FZ = 61 - klog;
  // N runs in int128 with 40 more fraction bits, so its precision is relative to its own size
  // rather than to max weight x max |v|; the written partial takes the unit that its magnitude
  // allows (below)
  const int FN = FZ + 40;
  int32_t R[RPT];
  int32_t Tlo[RPT];  // lowest floor(t) of the row's keys in this split
  int64_t Z[RPT];
  i128 N[RPT];
  uint64_t Zerr[RPT];
  u128 Nerr[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    R[i] = R_EMPTY;
    Tlo[i] = INT32_MAX;
    Z[i] = 0;
    N[i] = 0;
    Zerr[i] = 0;
    Nerr[i] = 0;
  }
  int32_t vec = INT32_MIN;  // this channel's VE as last applied to N

  if (warp >= NWARPS / 2) {
    // ======================= producer warpgroups: slicing and the score MMAs =======================
    const int ptid = tid - THREADS / 2, pwarp = warp - NWARPS / 2;
    bool rk_pending = ntiles > 0, rv_pending = ntiles > 0;
    uint32_t rk_ph = 0, rv_ph = 0;  // phase of the fetch in flight
    int par = 0;
    EA_PTW_INIT
    for (int i = 0; i < ntiles; ++i, par ^= 1) {
      const int64_t j0 = kbeg + (int64_t)i * BK;
      const int nvalid = (int)min((int64_t)BK, kend - j0);
      const uint32_t ph = (uint32_t)i & 1u, php = (uint32_t)(i - 1) & 1u;
      // the next tile's page-table entries, read now for its fetches below
      const int64_t pref = pwarp >= NWARPS / 2 - 2 ? page_ahead(P, row0, j0 + BK, kend) : -1;
      // ---- K(i): needs its raw rows, and pass 1 of tile i - 1 done with the digits, the lossy
      //      masks and the score accumulators ----
      bool okw = tc::mbar_wait(&S.bar_rk, ph, P.wait_debug);
      if (i > 0) okw &= tc::mbar_wait(&S.bar_p1, php, P.wait_debug);
      if (!group_sync_and(2, okw)) {
        ok_wait = false;
        break;
      }
      rk_pending = false;
      EA_PTW(THREADS / 2, 0)
#pragma unroll 1
      for (int it = 0; it < 2; ++it) {
        const int key = 64 * it + (ptid >> 2), l4 = ptid & 3;
        const bool valid = key < nvalid;
        const int rot = (l4 >> 1) + 2 * (key & 1);
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 a = make_uint4(0u, 0u, 0u, 0u);
          if (valid) a = *(const uint4*)(rawk + key * (D * 2) + l4 * 64 + 16 * ((j + rot) & 3));
          w[4 * j] = a.x;
          w[4 * j + 1] = a.y;
          w[4 * j + 2] = a.z;
          w[4 * j + 3] = a.w;
        }
        uint32_t mx = 0, mk = NZ_NONE;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const uint32_t m = w[q] & 0x7FFF7FFFu;
          mx = __vmaxu2(mx, m);
          mk = __vmins2(mk, nz_key(m));
        }
        mx = max(mx & 0xFFFFu, mx >> 16);
        int32_t mn = nz_key_min(mk);
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
          mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        }
        const int bad = mx >= 0x7F80u;
        const int lead = (mx == 0 || bad) ? INT32_MIN : lead_of_bits(mx);
        const int lsb = lead == INT32_MIN ? 0 : lead + 1 - P.W;
        const int ebase = lsb + 134;  // an element with exponent field E >= ebase loses no bits
        const bool fast = lead == INT32_MIN || (lsb >= -126 && lsb <= 126 &&
                                                (mn == 32767 || nz_key_mag(mn) >= ((uint32_t)ebase << 7)));
        const float sc = scale_of(max(-126, min(126, lsb)));
        uint32_t lm = 0;  // lossy elements, bit = dim - 32 l4
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int cj = (j + rot) & 3;
          uint32_t xs[8];
          if (lead == INT32_MIN) {
#pragma unroll
            for (int e = 0; e < 8; ++e) xs[e] = 0u;
          } else if (fast) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              xs[2 * q] = fixf_lo(w[4 * j + q], sc);
              xs[2 * q + 1] = fixf_hi(w[4 * j + q], sc);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const uint32_t b = (w[4 * j + (e >> 1)] >> (16 * (e & 1))) & 0xFFFFu;
              int lost = 0, b2 = 0;
              xs[e] = (uint32_t)fixq(b, lsb, lost, b2);
              lm |= (uint32_t)(lost != 0) << (8 * cj + e);
            }
          }
          uint32_t p0a, p1a, p2a, p3a, p0b, p1b, p2b, p3b;
          transpose4(xs[0], xs[1], xs[2], xs[3], p0a, p1a, p2a, p3a);
          transpose4(xs[4], xs[5], xs[6], xs[7], p0b, p1b, p2b, p3b);
          const uint32_t off = tc::kmajor_off(key, 32 * l4 + 8 * cj, BK);
          *(uint2*)(sK + 0 * K_PLANE + off) = make_uint2(p0a, p0b);
          *(uint2*)(sK + 1 * K_PLANE + off) = make_uint2(p1a, p1b);
          *(uint2*)(sK + 2 * K_PLANE + off) = make_uint2(p2a, p2b);
          *(uint2*)(sK + 3 * K_PLANE + off) = make_uint2(p3a, p3b);
        }
        S.klossy[key][l4] = lm;
        if (l4 == 0) {
          S.klsb[key] = lsb;
          S.kbad[key] = valid && bad;
        }
      }
      tc::fence_async_smem();
      group_sync(2);
      EA_PTW(THREADS / 2, 1)
      // score MMAs of tile i (the accumulators are free: pass 1 of tile i - 1 is done). Key digit t
      // goes to its own accumulator and is issued by lane 0 of producer warp t: an issuing thread
      // waits while the tensor core takes its operands, so four issuers share that wait.
      if (lane == 0 && pwarp < NK) {
        const int t = pwarp;
        tc::fence_after_sync();
        // descriptors: the base ones, then constant start-address offsets (16-byte units)
        constexpr uint32_t lbo_a = (BK / 8) * 128, lbo_b = (NSQ / 8) * 128;
        const uint64_t ad0 = tc::smem_desc(tc::smem_u32(sK + t * K_PLANE), lbo_a, 128);
        const uint64_t bd0 = tc::smem_desc(tc::smem_u32(sQ), lbo_b, 128);
        const uint32_t idesc = tc::idesc_i8(128, NSQ, t == NK - 1, true);
#pragma unroll
        for (int ks = 0; ks < D / 32; ++ks)
          tc::mma_i8(tmem + 32 * t, ad0 + ((ks * 2 * lbo_a) >> 4), bd0 + ((ks * 2 * lbo_b) >> 4), idesc, ks > 0);
        tc::mma_commit(tc::smem_u32(&S.bar_smma));
      }
      // the raw K rows are consumed: fetch the next tile's
      if (pwarp == NWARPS / 2 - 1 && i + 1 < ntiles) {
        tc::fence_async_smem();
        fetch_rows(P, P.k, row0, kvbase, j0 + BK, (int)min((int64_t)BK, kend - j0 - BK), rawk, &S.bar_rk, pref);
      }
      if (i + 1 < ntiles) {
        rk_pending = true;
        rk_ph = (uint32_t)(i + 1) & 1u;
      }

      // ---- V(i): needs its raw rows, and the P.V MMAs of tile i - 1 done with the value digits. The
      //      channel data of tile i - 1 stay in the other parity buffer until the consumers' merge;
      //      the P.V MMAs of tile i + 1 (after that merge) gate the next rewrite of this one ----
      okw = tc::mbar_wait(&S.bar_rv, ph, P.wait_debug);
      if (i > 0) okw &= tc::mbar_wait(&S.bar_pv, php, P.wait_debug);
      if (!group_sync_and(2, okw)) {
        ok_wait = false;
        break;
      }
      rv_pending = false;
      EA_PTW(THREADS / 2, 2)
      const int cp = ptid & 63, kq = ptid >> 6;
      const uint8_t* vsrc = rawv + (32 * kq) * (DV * 2) + cp * 4;  // word of key 32 kq + jj at jj * 256
      const int nv = min(32, max(0, nvalid - 32 * kq));             // this thread's valid keys
      uint32_t vmn;  // per channel (half) the key of the smallest nonzero |v| over this thread's keys
      {
        uint32_t mx = 0;
        vmn = NZ_NONE;
        if (nv == 32) {  // a full key quarter: no bounds test per load
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const uint32_t m = *(const uint32_t*)(vsrc + jj * (DV * 2)) & 0x7FFF7FFFu;
            mx = __vmaxu2(mx, m);
            vmn = __vmins2(vmn, nz_key(m));
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const uint32_t m = (jj < nv ? *(const uint32_t*)(vsrc + jj * (DV * 2)) : 0u) & 0x7FFF7FFFu;
            mx = __vmaxu2(mx, m);
            vmn = __vmins2(vmn, nz_key(m));
          }
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t m = (mx >> (16 * hh)) & 0xFFFFu;
          if (m >= 0x7F80u) {
            // a NaN / inf value: a domain error for the rows that see its key; the channel's range
            // comes from the finite values (the rows that do not see it use them)
            m = 0;
#pragma unroll 1
            for (int jj = 0; jj < nv; ++jj) {
              const uint32_t e = (*(const uint32_t*)(vsrc + jj * (DV * 2)) >> (16 * hh)) & 0x7FFFu;
              if (e >= 0x7F80u) {
                for (int g = 0; g < nrows; ++g)
                  if (S.rows[g] >= 0 && j0 + 32 * kq + jj < S.len[g]) atomicMax(&S.rst[g], ST_DOMAIN);
              } else {
                m = max(m, e);
              }
            }
          }
          S.ve4[kq][2 * cp + hh] = (int16_t)(m == 0 ? INT16_MIN : lead_of_bits(m) + 1);
        }
      }
      if (ptid < DV) {
        S.vl_n[par][ptid] = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) S.vlmask[par][ptid][q] = 0;
      }
      group_sync(2);
      EA_PTW(THREADS / 2, 3)
      // Digits of x = trunc(v 2^-lsb) through fp32 for every value. The values that lose bits (their
      // exponent field below ebase = lsb + 134) go to the channel's correction list, which adds back
      // exactly what the truncation dropped, or past its capacity to the bound. A channel whose
      // maximum lies at the very bottom of the bf16 range (lsb < -126) keeps no digits and is bounded.
      {
        int ebase2[2], lsb2[2];
        uint32_t keep2[2];
        float sc2[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          // running channel exponent: the previous tiles' and this tile's key quarters
          int ve = S.ve[par ^ 1][2 * cp + hh];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (S.ve4[q][2 * cp + hh] != INT16_MIN) ve = max(ve, (int)S.ve4[q][2 * cp + hh]);
          if (kq == 0) S.ve[par][2 * cp + hh] = ve;
          lsb2[hh] = ve == INT32_MIN ? 0 : ve - FV;
          const bool in_range = ve == INT32_MIN || lsb2[hh] >= -126;  // lsb <= 127 - 31 always
          ebase2[hh] = lsb2[hh] + 134;
          keep2[hh] = in_range ? 0xFFFFFFFFu : 0u;
          sc2[hh] = scale_of(in_range ? lsb2[hh] : 0);
        }
        const bool plain = nv == 32 && (keep2[0] & keep2[1]) != 0u;
#pragma unroll 1
        for (int q4 = 0; q4 < 2; ++q4) {
          uint32_t xa[16], xb[16];
          if (plain) {  // the usual case: 32 valid keys, both channels keep digits
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const uint32_t w = *(const uint32_t*)(vsrc + (16 * q4 + jj) * (DV * 2));
              xa[jj] = fixf_lo(w, sc2[0]);
              xb[jj] = fixf_hi(w, sc2[1]);
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int kk = 16 * q4 + jj;
              const uint32_t w = kk < nv ? *(const uint32_t*)(vsrc + kk * (DV * 2)) : 0u;
              xa[jj] = fixf_lo(w, sc2[0]) & keep2[0];
              xb[jj] = fixf_hi(w, sc2[1]) & keep2[1];
            }
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t* x = hh ? xb : xa;
            uint32_t pw[NV][4];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
              transpose4(x[4 * c4], x[4 * c4 + 1], x[4 * c4 + 2], x[4 * c4 + 3], pw[0][c4], pw[1][c4], pw[2][c4],
                         pw[3][c4]);
#pragma unroll
            for (int p = 0; p < NV; ++p)
              *(uint4*)(sV + p * V_PLANE + tc::kmajor_off(2 * cp + hh, 32 * kq + 16 * q4, BK)) =
                  make_uint4(pw[p][0], pw[p][1], pw[p][2], pw[p][3]);
          }
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int cc = 2 * cp + hh;
          const uint32_t thr = keep2[hh] ? ((uint32_t)max(ebase2[hh], 0) << 7) : 0x8000u;  // all, when bounded
          const int32_t mk = (int32_t)(int16_t)((vmn >> (16 * hh)) & 0xFFFFu);
          uint32_t lossy = 0;
          if (mk != 32767 && nz_key_mag(mk) < thr) {
#pragma unroll 1
            for (int jj = 0; jj < nv; ++jj) {
              const uint32_t b = (*(const uint32_t*)(vsrc + jj * (DV * 2)) >> (16 * hh)) & 0xFFFFu;
              const uint32_t mg = b & 0x7FFFu;
              if (mg == 0 || mg >= thr) continue;
              lossy |= 1u << jj;
              if (!keep2[hh]) continue;
              int lost2 = 0;
              const int32_t dx = lost_part24(b, lsb2[hh], lost2);
              const uint32_t k = atomicAdd(&S.vl_n[par][cc], 1u);
              if (k < VLCAP) {
                S.vl_k[par][cc][k] = (uint16_t)((32 * kq + jj) | (lost2 << 8));
                S.vl_dx[par][cc][k] = dx;
              }
            }
            if (!keep2[hh] && lossy) atomicAdd(&S.vl_n[par][cc], VL_BOUNDED);  // the whole channel is bounded
          }
          S.vlmask[par][cc][kq] = lossy;
        }
      }
      tc::fence_async_smem();
      group_sync(2);
      EA_PTW(THREADS / 2, 4)
      if (ptid == 0) mbar_arrive(&S.bar_vready);  // value digits and channel data of tile i
      // the raw V rows are consumed: fetch the next tile's
      if (pwarp == NWARPS / 2 - 2 && i + 1 < ntiles) {
        tc::fence_async_smem();
        fetch_rows(P, P.v, row0, kvbase, j0 + BK, (int)min((int64_t)BK, kend - j0 - BK), rawv, &S.bar_rv, pref);
      }
      if (i + 1 < ntiles) {
        rv_pending = true;
        rv_ph = (uint32_t)(i + 1) & 1u;
      }
    }
    EA_PTW_FLUSH(THREADS / 2)
    if (!ok_wait) S.abort = 1;
    // a wait that gave up: the copies still in flight get another bounded wait before the shared
    // memory is released
    if (rk_pending) tc::mbar_wait(&S.bar_rk, rk_ph, P.wait_debug);
    if (rv_pending) tc::mbar_wait(&S.bar_rv, rv_ph, P.wait_debug);
  } else {
    // ======================= consumer warpgroups: logits, weights, P.V, merges =======================
    const uint32_t tlane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    int par = 0;
    bool pv_pending = false;
    uint32_t pv_ph = 0;
    EA_PT_INIT
    for (int i = 0; i < ntiles; ++i, par ^= 1) {
      const int64_t j0 = kbeg + (int64_t)i * BK;
      const int nvalid = (int)min((int64_t)BK, kend - j0);
      const uint32_t ph = (uint32_t)i & 1u;
      {
        const bool okw = tc::mbar_wait(&S.bar_smma, ph, P.wait_debug);  // the score MMAs of tile i
        if (!group_sync_and(1, okw && !*(volatile int*)&S.abort)) {
          ok_wait = false;
          break;
        }
      }
      tc::fence_after_sync();
      EA_PT(0)
      // ---------------- pass 1: certified logits (lane: key; rows h, h + NWGC, ..) ----------------
      bool unc = false;
      {
        const int key = c;
        const bool klossy = (S.klossy[key][0] | S.klossy[key][1] | S.klossy[key][2] | S.klossy[key][3]) != 0;
        const bool kbad = S.kbad[key];
#pragma unroll 1
        for (int g = h; g < nrows; g += NWGC) {
          uint32_t dg[NK][4];
#pragma unroll
          for (int t = 0; t < NK; ++t) tc::tmem_ld4(tlane + 32 * t + 4 * g, dg[t]);
          tc::tmem_wait_ld();
          uint32_t out = T_MASKED;
          if (key < nvalid && j0 + key < S.len[g] && S.rows[g] >= 0) {
            if (kbad) {
              atomicMax(&S.rst[g], ST_DOMAIN);
            } else {
              // digit products (t, s) grouped by t + s: G_k = sum_{t + s = k} dg[t][s]
              const int32_t G0 = (int32_t)dg[0][0];
              const int32_t G1 = (int32_t)dg[0][1] + (int32_t)dg[1][0];
              const int32_t G2 = (int32_t)dg[0][2] + (int32_t)dg[1][1] + (int32_t)dg[2][0];
              const int32_t G3 = (int32_t)dg[0][3] + (int32_t)dg[1][2] + (int32_t)dg[2][1] + (int32_t)dg[3][0];
              const int32_t G4 = (int32_t)dg[1][3] + (int32_t)dg[2][2] + (int32_t)dg[3][1];
              const int32_t G5 = (int32_t)dg[2][3] + (int32_t)dg[3][2];
              const int32_t G6 = (int32_t)dg[3][3];
              const uint32_t lo4[4] = {(uint32_t)G0, (uint32_t)G1, (uint32_t)G2, (uint32_t)G3};
              const uint32_t hi3[3] = {(uint32_t)G4, (uint32_t)G5, (uint32_t)G6};
              const int64_t acc = recomb<4>(lo4) + (int64_t)((uint64_t)recomb<3>(hi3) << 32);
              const bool qlossy = (S.qlossy[g][0] | S.qlossy[g][1] | S.qlossy[g][2] | S.qlossy[g][3]) != 0;
              const int sexp = S.qlsb[g] + S.klsb[key];
              uint32_t fb;
              bool done = false, differ = false;
              uint64_t err = 0;
              if (qlossy || klossy) {
                // |q k - Q K| <= |dq| |k| + |Q| |dk| over the lossy elements (units 2^(qlsb + klsb))
                for (int wd = 0; wd < 4; ++wd) {
                  const uint32_t ql = S.qlossy[g][wd], kl = S.klossy[key][wd];
                  for (uint32_t m = ql; m; m &= m - 1) {
                    const int ii = 32 * wd + __ffs(m) - 1;
                    const int32_t kf = read_fix(sK, K_PLANE, key, ii, BK);
                    err += (uint64_t)(kf < 0 ? -kf : kf) + ((kl >> (ii & 31)) & 1u);
                  }
                  for (uint32_t m = kl; m; m &= m - 1) {
                    const int ii = 32 * wd + __ffs(m) - 1;
                    const int32_t qf = q_fix(sQ, g, ii);
                    err += (uint64_t)(qf < 0 ? -qf : qf);
                  }
                }
                done = f64::logit_interval_f64(acc, err, sexp, am_d, P.ae, fb, differ);
              } else {
                done = f64::logit_f64(acc, sexp, am_d, P.ae, fb);
              }
              // the binary64 fast path first; the integer evaluation decides what it cannot certify
              if (done) {
                out = fb;
              } else if (differ) {
                out = T_UNCERT;
              } else {
                Rnd t = rnd_zero();
                const int ls = (qlossy || klossy) ? logit_bounded(acc, err, sexp, P.am, P.ae, t)
                                                  : logit_exact64(acc, sexp, P.am, P.ae, t);
                if (ls == LOGIT_OK) out = rnd_to_f32_bits(t);
                else if (ls == LOGIT_UNCERTIFIED) out = T_UNCERT;
                else atomicMax(&S.rst[g], ST_DOMAIN);
              }
            }
          }
          sT[g * BK + key] = out;
          // tile bound of the certified logits: w = RN24(2^t) <= 2^(floor(t) + 1) < 2^(ceil(t) + 1)
          const float tf = __uint_as_float(out);
          int32_t rl = INT32_MIN, ll = INT32_MAX;
          if (out != T_MASKED && out != T_UNCERT && fabsf(tf) < 1073741824.0f) {
            rl = __float2int_ru(tf) + 1;
            ll = __float2int_rd(tf);
          }
          rl = __reduce_max_sync(0xffffffffu, rl);
          ll = __reduce_min_sync(0xffffffffu, ll);
          if (lane == 0) {
            S.rt[warp & 3][g] = rl;
            S.rtlo[warp & 3][g] = ll;
          }
          unc |= out == T_UNCERT;
        }
      }
      tc::fence_before_sync();
      const bool any_unc = group_sync_or(1, unc);
      if (tid == 0) mbar_arrive(&S.bar_p1);  // the key digits, masks and score accumulators are free
      EA_PT(1)
      // ---------------- exact scores of the uncertified pairs, one warp per pair ----------------
      if (any_unc) {
        for (int e0 = 0; e0 < nrows * BK; e0 += THREADS / 2) {
          const int e = e0 + warp * 32 + lane;
          const uint32_t hit = __ballot_sync(0xffffffffu, e < nrows * BK && sT[e] == T_UNCERT);
          for (uint32_t m = hit; m; m &= m - 1) {
            const int ee = e0 + warp * 32 + __ffs(m) - 1;
            const int g = ee / BK, key = ee % BK;
            int64_t run;
            const int64_t kr = run_start(P, row0, j0 + key, run);
            Rnd t = rnd_zero();
            const int ls = warp_exact_logit(P.q, P.k, P.am, P.ae, S.rows[g], kr, t);
            if (lane == 0) {
              if (ls == LOGIT_OK) {
                sT[ee] = rnd_to_f32_bits(t);
              } else {
                sT[ee] = T_MASKED;
                atomicMax(&S.rst[g], ST_DOMAIN);
              }
              ++n_exact;
            }
          }
        }
        group_sync(1);
        // the tile bounds again, now over the exact logits too
#pragma unroll 1
        for (int g = h; g < nrows; g += NWGC) {
          const uint32_t tb = sT[g * BK + c];
          const float tf = __uint_as_float(tb);
          int32_t rl = INT32_MIN, ll = INT32_MAX;
          if (tb != T_MASKED && fabsf(tf) < 1073741824.0f) {
            rl = __float2int_ru(tf) + 1;
            ll = __float2int_rd(tf);
          }
          rl = __reduce_max_sync(0xffffffffu, rl);
          ll = __reduce_min_sync(0xffffffffu, ll);
          if (lane == 0) {
            S.rt[warp & 3][g] = rl;
            S.rtlo[warp & 3][g] = ll;
          }
        }
        group_sync(1);
      }
      EA_PT(2)
      // ---------------- pass 2: weights, W digits ----------------
#pragma unroll 1
      for (int g = h; g < nrows; g += NWGC) {
        const int key = c;
        const int32_t Rt = max(max(S.rt[0][g], S.rt[1][g]), max(S.rt[2][g], S.rt[3][g]));
        const uint32_t tb = sT[g * BK + key];
        uint64_t W = 0;
        uint32_t lw = 0;
        if (tb != T_MASKED && Rt != INT32_MIN) {
          uint32_t M;
          int64_t E;
          int ws = W_OK;
          const float tf = __uint_as_float(tb);
          int32_t Ef;
          // w < 2^(t + 1) <= 2^(Rt - 48): W = 0, a truncated (nonzero) weight
          const bool tiny = tf > -1073741824.0f && (double)tf < (double)Rt - 49.0;
          if (tiny) {
            M = 0;
            E = 0;
          } else if (f64::weight_f64(tb, S.td, M, Ef)) {
            E = Ef;
          } else {
            // (separate variables for the out-of-line call: M and E keep no address)
            const Rnd t = rnd_from_f32(tb);
            uint32_t Mi;
            int64_t Ei;
            ws = weight_from_logit(t, g_ta64, g_tb64, Mi, Ei);
            if (ws == W_RISKY) {
              ++n_wide;
              ws = wide_weight(t, Mi, Ei);
            }
            M = Mi;
            E = Ei;
          }
          if (ws != W_OK) {
            atomicMax(&S.rst[g], ST_TIER3);  // |t| >= 2^30 or a still-risky weight
          } else if (tiny) {
            lw = 1;
          } else {
            const int sh = (int)(E + FW - Rt);
            if (sh >= 0) {
              W = (uint64_t)M << sh;
            } else if (sh > -64) {
              W = (uint64_t)M >> (-sh);
              lw = (W << (-sh)) != M;
            } else {
              lw = 1;
            }
          }
        }
#pragma unroll
        for (int wd = 0; wd < NW; ++wd) sW[tc::kmajor_off(6 * g + wd, key, NSW)] = (uint8_t)(W >> (8 * wd));
        const uint64_t zs = warp_sum_u64(W);
        const uint32_t zl = __reduce_add_sync(0xffffffffu, lw);
        if (lane == 0) {
          S.zs[warp & 3][g] = zs;
          S.zl[warp & 3][g] = zl;
        }
      }
      tc::fence_async_smem();
      bool okw = tc::mbar_wait(&S.bar_vready, ph, P.wait_debug);  // the producers' value digits of tile i
      if (!group_sync_and(1, okw)) {
        ok_wait = false;
        break;
      }
      EA_PT(3)
      // ---------------- P.V MMAs: 4 value digits x (N = 48: row weight digits) ----------------
      // value digit u to its own accumulator, issued by lane 0 of consumer warp u
      if (lane == 0 && warp < NV) {
        const int u = warp;
        tc::fence_after_sync();
        constexpr uint32_t lbo_a = (DV / 8) * 128, lbo_b = (NSW / 8) * 128;
        const uint64_t ad0 = tc::smem_desc(tc::smem_u32(sV + u * V_PLANE), lbo_a, 128);
        const uint64_t bd0 = tc::smem_desc(tc::smem_u32(sW), lbo_b, 128);
        const uint32_t idesc = tc::idesc_i8(128, NSW, u == NV - 1, false);
#pragma unroll
        for (int ks = 0; ks < BK / 32; ++ks)
          tc::mma_i8(tmem + COL_O + NSW * u, ad0 + ((ks * 2 * lbo_a) >> 4), bd0 + ((ks * 2 * lbo_b) >> 4), idesc,
                     ks > 0);
        tc::mma_commit(tc::smem_u32(&S.bar_pv));
      }
      pv_pending = true;
      pv_ph = ph;
      EA_PT(7)
      // meanwhile: this channel's exponent change, the rows' merges and bounds (registers only)
      const int ve_now = S.ve[par][c];
      int sh_base[RPT];
#pragma unroll
      for (int ii = 0; ii < RPT; ++ii) {
        const int g = h + NWGC * ii;
        sh_base[ii] = INT32_MIN;
        if (g >= nrows) continue;
        if (ve_now != vec && vec != INT32_MIN) {  // VE_c grew: N in the coarser unit
          const int d = ve_now - vec;
          N[ii] = shift_floor128(N[ii], -d);
          Nerr[ii] = scale_ceil128(Nerr[ii], -d) + 1;
        }
        const int32_t Rt = max(max(S.rt[0][g], S.rt[1][g]), max(S.rt[2][g], S.rt[3][g]));
        if (Rt == INT32_MIN) continue;
        Tlo[ii] = min(Tlo[ii], min(min(S.rtlo[0][g], S.rtlo[1][g]), min(S.rtlo[2][g], S.rtlo[3][g])));
        const int32_t Rn = R[ii] == R_EMPTY ? Rt : max(R[ii], Rt);
        if (R[ii] != R_EMPTY && Rn > R[ii]) {
          const int d = Rn - R[ii];
          N[ii] = shift_floor128(N[ii], -d);
          Nerr[ii] = scale_ceil128(Nerr[ii], -d) + 1;
          int lost;
          Z[ii] = floor_shift(Z[ii], -d, lost);
          Zerr[ii] = scale_ceil(Zerr[ii], -d) + (uint64_t)lost;
        }
        R[ii] = Rn;
        const uint64_t zt = S.zs[0][g] + S.zs[1][g] + S.zs[2][g] + S.zs[3][g];
        const uint64_t nlw = (uint64_t)S.zl[0][g] + S.zl[1][g] + S.zl[2][g] + S.zl[3][g];
        const int zsh = (Rt - FW) - (Rn - FZ);
        int lost = 0;
        Z[ii] += floor_shift((int64_t)zt, zsh, lost);
        Zerr[ii] += scale_ceil(nlw, zsh) + (uint64_t)lost;
        const int sb = (Rt - FW - FV) - (Rn - FN);
        sh_base[ii] = sb;
        Nerr[ii] += scale_ceil128(nlw, sb + FV);  // truncated weights: < 1 W unit times |v| < 2^VE_c
        // values that lost bits in the V window: their lost parts times the weights, added exactly up
        // to a floor (units 2^(sb - 24)); beyond the list's capacity, the bound of < W + 1 W units
        // times one V unit per such value
        const uint32_t nl = S.vl_n[par][c];
        if (nl <= VLCAP) {
          i128 corr = 0;
          u128 cerr = 0;
#pragma unroll 1
          for (uint32_t k = 0; k < nl; ++k) {
            const uint32_t ck = S.vl_k[par][c][k];
            const int key = (int)(ck & 0xFFu);
            uint64_t W = 0;
#pragma unroll
            for (int wd = 0; wd < NW; ++wd) W |= (uint64_t)sW[tc::kmajor_off(6 * g + wd, key, NSW)] << (8 * wd);
            corr += shift_floor128((i128)(int64_t)W * S.vl_dx[par][c][k], sb - 24);  // |W dx| < 2^72
            cerr += (sb - 24 < 0) ? 1u : 0u;
            if ((ck >> 8) & 1u) cerr += scale_ceil128((u128)W + 1, sb - 24);
          }
          N[ii] += corr;
          Nerr[ii] += cerr;
        } else {
          uint64_t vw = 0;
#pragma unroll 1
          for (int q4 = 0; q4 < 4; ++q4)
            for (uint32_t m = S.vlmask[par][c][q4]; m; m &= m - 1) {
              const int key = 32 * q4 + __ffs(m) - 1;
              uint64_t W = 0;
#pragma unroll
              for (int wd = 0; wd < NW; ++wd) W |= (uint64_t)sW[tc::kmajor_off(6 * g + wd, key, NSW)] << (8 * wd);
              vw += W + 1;
            }
          // a truncated value lost < 1 V unit; a bounded channel's values are < 2^VE_c: 2^FV units
          Nerr[ii] += scale_ceil128(vw, sb + (nl >= VL_BOUNDED ? FV : 0));
        }
        Nerr[ii] += (sb < 0) + (24 + sb < 0) + (48 + sb < 0);  // floors of the three round shifts
      }
      vec = ve_now;
      EA_PT(4)
      // each thread waits; after a wait that gave up the drain reads stale TMEM and the vote at
      // the end of the tile drops it
      const bool ok_pv = tc::mbar_wait(&S.bar_pv, ph, P.wait_debug);
      tc::fence_after_sync();
      EA_PT(5)
      // ---------------- drain: N[g][c] += sum_k 2^(8k) G_k, G_k = sum_{u + w = k} D_u[w] ----------------
#pragma unroll
      for (int ii = 0; ii < RPT; ++ii) {
        const int g = h + NWGC * ii;
        if (g >= nrows) break;  // uniform across the warp
        uint32_t d0[8], d1[8], d2[8], d3[8];
        tc::tmem_ld8(tlane + COL_O + 6 * g, d0);
        tc::tmem_ld8(tlane + COL_O + NSW + 6 * g, d1);
        tc::tmem_ld8(tlane + COL_O + 2 * NSW + 6 * g, d2);
        tc::tmem_ld8(tlane + COL_O + 3 * NSW + 6 * g, d3);
        tc::tmem_wait_ld();
        if (sh_base[ii] == INT32_MIN) continue;
        // |D_u[w]| < 128 keys x 255 x 255 < 2^23, so each group (<= 4 terms) fits int32
        const int32_t s0 = (int32_t)d0[0];
        const int32_t s1 = (int32_t)d0[1] + (int32_t)d1[0];
        const int32_t s2 = (int32_t)d0[2] + (int32_t)d1[1] + (int32_t)d2[0];
        const int32_t s3 = (int32_t)d0[3] + (int32_t)d1[2] + (int32_t)d2[1] + (int32_t)d3[0];
        const int32_t s4 = (int32_t)d0[4] + (int32_t)d1[3] + (int32_t)d2[2] + (int32_t)d3[1];
        const int32_t s5 = (int32_t)d0[5] + (int32_t)d1[4] + (int32_t)d2[3] + (int32_t)d3[2];
        const int32_t s6 = (int32_t)d1[5] + (int32_t)d2[4] + (int32_t)d3[3];
        const int32_t s7 = (int32_t)d2[5] + (int32_t)d3[4];
        const int32_t s8 = (int32_t)d3[5];
        const uint32_t r0[3] = {(uint32_t)s0, (uint32_t)s1, (uint32_t)s2};
        const uint32_t r1[3] = {(uint32_t)s3, (uint32_t)s4, (uint32_t)s5};
        const uint32_t r2[3] = {(uint32_t)s6, (uint32_t)s7, (uint32_t)s8};
        const int sb = sh_base[ii];
        N[ii] += shift_floor128(recomb<3>(r0), sb) + shift_floor128(recomb<3>(r1), 24 + sb) +
                 shift_floor128(recomb<3>(r2), 48 + sb);
      }
      tc::fence_before_sync();
      if (!group_sync_and(1, ok_pv)) {
        ok_wait = false;
        break;
      }
      pv_pending = false;
      EA_PT(6)
    }
    EA_PT_FLUSH
    if (!ok_wait) S.abort = 1;
    if (pv_pending) tc::mbar_wait(&S.bar_pv, pv_ph, P.wait_debug);
    n_exact = __reduce_add_sync(0xffffffffu, n_exact);
    n_wide = __reduce_add_sync(0xffffffffu, n_wide);
    if (lane == 0) {
      stat_add(P, STAT_SCORE_EXACT, n_exact);
      stat_add(P, STAT_WEIGHT_WIDE, n_wide);
    }
  }
  tc::fence_before_sync();
  __syncthreads();  // both roles are done: row status (also set by the producers) is final
  // ---------------- split partials of this CTA's rows (after both roles are done) ----------------
  if (warp < NWARPS / 2) {
#pragma unroll
    for (int ii = 0; ii < RPT; ++ii) {
      const int g = h + NWGC * ii;
      if (g >= nrows) break;
      const int32_t row = S.rows[g];
      if (row < 0) continue;
      const int64_t pi = (int64_t)split * P.rows + row;
      int st = S.abort ? ST_TIER3 : S.rst[g];
      // logits spanning more than SPREAD_CHECK below the bound: tier 3 decides the reference's
      // exponent-spread rule
      if (st == ST_OK && R[ii] != R_EMPTY && Tlo[ii] != INT32_MAX && (int64_t)R[ii] - Tlo[ii] > SPREAD_CHECK)
        st = ST_TIER3;
      if (c == 0) {
        const int dsh = FZ - P.FZ;
        const int64_t zlo = shift_floor(Z[ii], -dsh);
        const int64_t zhi = -shift_floor(-(Z[ii] + (int64_t)Zerr[ii]), -dsh);
        P.pR[pi] = R[ii];
        P.pZ[pi] = zlo;
        P.pZe[pi] = (uint64_t)(zhi - zlo);
        P.pSt[pi] = st;
      }
      const bool empty = R[ii] == R_EMPTY || vec == INT32_MIN;
      // this kernel's N interval is [N - Nerr, N + Nerr] in units 2^(R + VE_c - FN); partials are
      // one-sided [N, N + Nerr] in units 2^(NR - P.FZ) with |N| < 2^(P.FZ + klog - 2) < (this
      // split's keys) 2^P.FZ, the bound the exact merge of partials relies on: take the finest unit
      // 2^s (s >= 0) that keeps the interval ends below it, floor the low end, ceil the high end
      const i128 lo = N[ii] - (i128)Nerr[ii], hi = N[ii] + (i128)Nerr[ii];
      const u128 mag = (u128)(lo < 0 ? -lo : lo) > (u128)(hi < 0 ? -hi : hi) ? (u128)(lo < 0 ? -lo : lo)
                                                                                : (u128)(hi < 0 ? -hi : hi);
      const int sx = max(0, bitlen128(mag) + 1 - (P.FZ + klog - 2));
      const int64_t nlo = (int64_t)shift_floor128(lo, -sx);
      const int64_t nhi = (int64_t)(-shift_floor128(-hi, -sx));
      P.pNR[pi * DV + c] = empty ? R_EMPTY : R[ii] + vec - FN + P.FZ + sx;
      P.pN[pi * DV + c] = empty ? 0 : nlo;
      P.pNe[pi * DV + c] = empty ? 0 : (uint64_t)(nhi - nlo);
    }
  }
  if (tid == 0) {
    unsigned long long pairs = 0;
    for (int g = 0; g < nrows; ++g) {
      const int64_t l = S.rows[g] >= 0 ? S.len[g] : 0;
      const int64_t a = kbeg, b = min(kend, l);
      if (b > a) pairs += (unsigned long long)(b - a);
    }
    stat_add(P, STAT_PAIRS, pairs);
    stat_add(P, STAT_TC_PAIRS, pairs);
    if (S.abort) stat_add(P, STAT_WAIT_EXPIRED, 1);  // a bounded wait gave up
  }
  if (warp == 0) tc::tmem_free(tmem, TMEM_COLS);
}

}  // namespace tcd

// Grid (segments, splits); writes split partials (P.pR ..) for every listed row. max_rows: the
// most rows any segment holds (1..8; 8 when unknown).
cudaError_t launch_tc_decode(const Prob& P, const int32_t* seg_rows, int64_t nseg, int max_rows, cudaStream_t st) {
  // the shared-memory opt-in is a property of the function on a device: set it once per device
  // (not per launch, so a launch inside a stream capture issues nothing but the kernel)
  static bool attr_set[64][3] = {};
  const int v = max_rows <= tcd::NWGC ? 0 : max_rows <= 2 * tcd::NWGC ? 1 : 2;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev][v]) {
    cudaError_t e = v == 0 ? cudaFuncSetAttribute(tcd::tc_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)tcd::SMEM_BYTES)
                    : v == 1 ? cudaFuncSetAttribute(tcd::tc_decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    (int)tcd::SMEM_BYTES)
                             : cudaFuncSetAttribute(tcd::tc_decode_kernel<tcd::RPT_MAX>,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tcd::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev][v] = true;
  }
  dim3 grid((unsigned)nseg, (unsigned)P.splits);
  if (v == 0)
    tcd::tc_decode_kernel<1><<<grid, tcd::THREADS, tcd::SMEM_BYTES, st>>>(P, seg_rows);
  else if (v == 1)
    tcd::tc_decode_kernel<2><<<grid, tcd::THREADS, tcd::SMEM_BYTES, st>>>(P, seg_rows);
  else
    tcd::tc_decode_kernel<tcd::RPT_MAX><<<grid, tcd::THREADS, tcd::SMEM_BYTES, st>>>(P, seg_rows);
  return cudaGetLastError();
}

}  // namespace ea

#ifdef EA_PHASE_TIMERS
// phase clocks of the decode kernel (timer builds only): copies and clears the 16 counters
extern "C" int ea_debug_phase_cycles_decode(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, ea::tcd::g_phase_cycles, sizeof(unsigned long long) * 16);
  unsigned long long z[16] = {0};
  return cudaMemcpyToSymbol(ea::tcd::g_phase_cycles, z, sizeof(z)) == cudaSuccess ? 0 : -4;
}
#endif
