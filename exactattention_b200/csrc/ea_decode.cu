// Tensor-core (tcgen05 / TMEM) tier-1 kernel of certified ExactAttention for decode: a few query
// rows (one GQA group of one sequence, at most 8) against a long key sequence, d = dv = 128.
//
// The prefill kernel puts 128 query rows on the MMA's M side; a decode group has 1-8 rows, so
// here the KEYS take the M side and the rows' digits go to N:
//   scores   S^T[key, (g, s)] = K_t . Q_s for key digit planes t (A, 128 keys x 128 dims, held in
//            TENSOR MEMORY: key r in TMEM lane r) against one B tile holding every row's 4 query
//            digit planes (N = 4 x rows). Query digits are balanced (signed bytes) so one B tile
//            has one signedness.
//   P.V      O^T[c, (g, w)] = V_u . W_w for value digit planes u (A, 128 channels x 128 keys, in
//            shared memory) against one B tile of every row's 6 weight digit planes (N = 6 x
//            rows); values in a 30-bit window against the channel's running maximum, as four
//            unsigned digits of x + 2^30 (a low byte and three OFFSET-BINARY bytes), the offset
//            removed exactly with the tile's weight sum.
// Digit products are grouped by digit position on the CUDA cores (int32 sums) and recombined
// exactly in int64 / int128, with the same fixed-point windows, bounds and certification as the
// prefill kernel. Each CTA takes one (segment, split): the split's 128-key tiles arrive by bulk
// copies (cp.async.bulk, completing on mbarriers) into two raw staging buffers per tensor, so
// the copies of tile i + 1 land while tile i is sliced. Every CTA writes its rows' split
// partials; the split combine merges them (any split count gives the same bits).
//
// Thread roles (512 threads, warp-specialised, one warp of each producer role per SM sub-
// partition so the roles overlap):
//   warps 8-11 (K producers): one key per thread, which is also the key's TMEM lane. The raw K
//     tile arrives through a 2D TMA tensor map as two 64-dimension halves of 128-byte rows with
//     the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r % 8)), so the 32 threads of
//     a warp read 32 rows without bank conflicts (page sizes that do not tile 128 keys take dense
//     bulk copies instead). Each thread turns its key into 4 digit planes (27-bit two's complement window,
//     exact through fp32), stores them into tensor memory and its warp's lane 0 issues the score
//     MMAs of one key digit plane (A from TMEM, B = the query digits in shared memory). It also
//     keeps the key's fixed-point values at the few dimensions where some query row lost bits
//     (the consumers' error bound), so the raw rows are free once sliced and the next tiles'
//     copies run two tiles ahead.
//   warps 12-15 (V producers): 4 channels x 32 keys per thread; value digits by round-toward-zero
//     fused multiply-adds (the scale and the conversion to offset-binary integer bits in one
//     instruction: one for the high three bytes, one on a clamped copy for the low byte, which
//     only values at the bottom of the window have).
//   warps 0-7 (consumers, the TMEM lane quadrant = warp % 4): logits, weights and W digits, the
//     P.V MMAs (lane 0 of warp u issues value digit plane u), the running sums (pass 1 / pass 2:
//     lane = key; drain: lane = channel; rows g = warp / 4 + 2 i).
// mbarriers carry the hand-offs (raw K / V landed per buffer, score MMAs done, pass 1 done, value
// digits ready, P.V done) and every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "ea_core.cuh"
#include "ea_fast64.cuh"
#include "ea_numerics.h"
#include "ea_tables.cuh"
#include "ea_tc_common.cuh"
#include "ea_tcgen05.cuh"

#include <cstring>

namespace ea {
namespace tcd {

using namespace tcc;

#ifdef EA_PHASE_TIMERS
__device__ unsigned long long g_phase_cycles[16];
// the counters live in the dynamic shared memory (no static shared memory moves its base)
#undef EA_PT_DECL
#define EA_PT_DECL                    \
  unsigned long long* ea_pt_acc = S.pt_acc; \
  if (threadIdx.x < 16) ea_pt_acc[threadIdx.x] = 0;
// K producers (thread 256) keep counters 8-11, V producers (their first thread) counters 12-15
#define EA_PTK_INIT long long ptk_last = clock64();
#define EA_PTK(i)                          \
  if (tid == 256) {                        \
    const long long pt_now = clock64();    \
    ea_pt_acc[8 + (i)] += pt_now - ptk_last; \
    ptk_last = pt_now;                     \
  }
#define EA_PTV_INIT long long ptv_last = clock64();
#define EA_PTV(i)                           \
  if (tid == VW0 * 32) {                    \
    const long long pt_now = clock64();     \
    ea_pt_acc[12 + (i)] += pt_now - ptv_last; \
    ptv_last = pt_now;                      \
  }
#define EA_PT_FLUSH_RANGE(who, lo, hi) \
  if (tid == (who))                    \
    for (int i = (lo); i < (hi); ++i) atomicAdd(&g_phase_cycles[i], ea_pt_acc[i]);
#else
#define EA_PTK_INIT
#define EA_PTK(i)
#define EA_PTV_INIT
#define EA_PTV(i)
#define EA_PT_FLUSH_RANGE(who, lo, hi)
#endif

constexpr int BK = 128, D = 128, DV = 128, GD = 8;
constexpr int NQ = 4, NK = 4, NW = 6, NV = 4;
constexpr int FW = 48, FV = 30;  // V: 30-bit window, 4 digits (very few values fall below it)
constexpr float V_MAGIC = 12582912.0f;  // 1.5 x 2^23: y + V_MAGIC has y + 2^22 in its low 23 bits
// warps: consumers 0 .. NC - 1, K producers NC .. NC + KW - 1, V producers the last four
template <int NC, int KW>
__host__ __device__ constexpr int threads_of() { return 32 * (NC + KW + 4); }
// registers a thread of each role keeps with 8 K producer warps (640 threads, 96 registers a
// thread at launch): the producer warpgroups give registers back to the consumers
constexpr int REG_CONSUMER = 120, REG_PRODUCER = 80, REG_LAUNCH = 96;
constexpr int REG_SPLIT = 256 * REG_CONSUMER + 384 * REG_PRODUCER;
constexpr uint32_t VLCAP = 2;
constexpr int NQL = 4;  // dimensions whose k values the K producers keep for the consumers' bound
constexpr uint32_t VL_BOUNDED = 1u << 20;  // marks a channel without digits (all values bounded)
constexpr uint32_t TMEM_COLS = 512;
constexpr int NSQ = NQ * GD;  // score B rows: n = 4 g + s
constexpr int NSW = NW * GD;  // P.V B rows: n = 6 g + w
// TMEM columns: K digit planes (A of the scores; plane t at COL_K + 32 t, 4 bytes a column),
// score accumulators (plane t at COL_S + 32 t + n), P.V accumulators (plane u at COL_O + 48 u + n).
// Segments of at most two rows (N = 8 score columns a plane) double-buffer the K digits and the
// score accumulators instead: K buffer b at 128 b, scores of buffer b at 256 + 32 b + 8 t + n,
// P.V accumulators at 320 + 48 u + n.
constexpr uint32_t COL_K = 0, COL_S = 128, COL_O = 256;
constexpr uint32_t DB_COL_S = 256, DB_COL_O = 320;
static_assert(COL_O + NV * NSW <= TMEM_COLS && DB_COL_O + NV * NSW <= TMEM_COLS, "tensor memory budget");

constexpr uint32_t RAWK_BUF = BK * D * 2;   // 32768: two swizzled halves of 128 x 128 bytes, or 128 dense rows
constexpr uint32_t KHALF = BK * 128;         // 16384
constexpr uint32_t RAWV_BUF = BK * DV * 2;   // 32768
constexpr uint32_t V_PLANE = DV * BK;            // 16384
constexpr uint32_t OFF_RAWK = 0;
constexpr uint32_t OFF_RAWV = OFF_RAWK + 2 * RAWK_BUF;
constexpr uint32_t OFF_V = OFF_RAWV + 2 * RAWV_BUF;
constexpr uint32_t OFF_Q = OFF_V + NV * V_PLANE;
constexpr uint32_t OFF_W = OFF_Q + NSQ * D;
constexpr uint32_t OFF_T = OFF_W + NSW * BK;
constexpr uint32_t OFF_SMALL = OFF_T + GD * BK * 4;

struct Small {
  // key metadata by tile parity (the K producers write tile i + 1's while the consumers read i's)
  uint32_t klossy[2][BK][4];
  int32_t kqv[2][BK][NQL];  // fixed-point k at the listed dimensions where some q row is lossy
  int16_t klsb[2][BK];
  uint8_t kbad[2][BK];
  // value metadata of the last two tiles (by tile parity): per channel, up to VLCAP values that
  // lost bits in the V window, with their lost parts (units 2^(lsb_c - 24), floored, >= 0), added
  // back exactly in the drain: (key | still-lossy << 8), part
  uint32_t vl_n[2][DV];
  uint16_t vl_k[2][DV][VLCAP];
  int32_t vl_dx[2][DV][VLCAP];
  int32_t ve[2][DV];   // running channel exponent VE_c (|v| < 2^VE_c so far), by tile parity
  int16_t ve4[2][DV];  // per key half maxima of the current tile (INT16_MIN: none)
  uint64_t td[256];    // binary64 2^(j/256) of the fast weight path
  uint32_t kscan[2][BK][2];  // with two K threads a key: each half's largest magnitude and nonzero-minimum key
  int64_t qsum[GD];    // per query row: the sum of its fixed-point elements (Toeplitz layout)
  int32_t qlk[NQL];    // the dimensions where some query row of the segment lost bits, ascending
  int32_t nqlk;        // their number, or -1 when there are more than NQL
  int32_t rows[GD];
  int32_t len[GD];
  int32_t qlsb[GD];
  int32_t rst[GD];
  uint32_t qlossy[GD][4];
  int32_t rt[4][GD];    // per lane quadrant
  int32_t rtlo[4][GD];  // lowest floor(t) per lane quadrant (the exponent-spread check)
  uint64_t zs[4][GD];
  uint32_t zl[4][GD];
  // raw K / V tiles landed (per buffer); score MMAs done; pass 1 done; value digits and channel
  // data ready; P.V MMAs done
  // (score MMAs / pass 1 by score buffer: one buffer, or two for double-buffered segments)
  uint64_t bar_rk[2], bar_rv[3], bar_smma[2], bar_p1[2], bar_vready, bar_pv;
  int32_t abort;  // a bounded wait gave up in some role
  uint32_t tmem;
#ifdef EA_PHASE_TIMERS
  unsigned long long pt_acc[16];
#endif
  int32_t nrows;
  int32_t maxlen;
  int32_t row0;
};

constexpr uint32_t SMEM_BYTES = OFF_SMALL + sizeof(Small);
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

// The Toeplitz layout (segments of at most two rows, 8 K producer warps). Every element stays one
// 32-bit word whose four bytes are its unsigned digits: a key element x (|x| < 2^27) as x + 2^27,
// a value element x (|x| < 2^30) as x + 2^30. An MMA's K dimension runs over (element, byte): key
// (or channel) r's A row holds its elements' words in tensor memory, one element a column. The B
// tiles hold the other operand's digits shifted per output column: score column (g, k) holds, at
// byte u of dimension i, query digit Q_(k-u)[g][i] (zero outside 0..3), so the accumulator of
// column k is the digit group G_k = sum_(t + s = k) K_t . Q_s (k = 0..6) and no byte transposes
// are needed on either side; the P.V tile likewise holds weight digit W_(k-u) at byte u of key j
// (k = 0..8). The biases come out exactly: 2^27 times the row's query sum, 2^30 times the tile's
// weight sum. B tiles use the 128-byte swizzle (conflict-free word stores).
// Shared memory: raw K staging as above, raw V staging in three buffers (V tiles fetched three
// ahead), score B tile (16 rows: n = 8 g + k), P.V B tile (32
// rows: n = 16 g + k), logits, the rows' fixed-point query elements and the tile's weights.
constexpr uint32_t T_QROWS = 16, T_WROWS = 32, T_KB = 512;  // B rows, K bytes of a B row
constexpr uint32_t T_OFF_QT = OFF_RAWV + 3 * RAWV_BUF;
constexpr uint32_t T_OFF_WT = T_OFF_QT + T_QROWS * T_KB;
constexpr uint32_t T_OFF_T = T_OFF_WT + T_WROWS * T_KB;
constexpr uint32_t T_OFF_QF = T_OFF_T + GD * BK * 4;
constexpr uint32_t T_OFF_WV = T_OFF_QF + 2 * D * 4;
// Lost parts of window elements (Toeplitz layout), for the exact correction of lossy scores: per
// tile parity, K thread half h and key, up to 2 elements (dimension, dk = k - K 2^klsb, exact in
// fp32) and their count (more than 2: the list is incomplete); per query row and listed lossy
// dimension n (S.qlk), dq = q - Q 2^qlsb (0 where the row lost nothing)
struct KcArea {
  float kcd[2][2][BK][2];
  uint8_t kci[2][2][BK][2];
  uint8_t kcn[2][2][BK];
  float qdq[2][NQL];
};
constexpr uint32_t T_OFF_KC = T_OFF_WV + 2 * BK * 8;
constexpr uint32_t T_OFF_SMALL = T_OFF_KC + (uint32_t)((sizeof(KcArea) + 15) / 16 * 16);
constexpr uint32_t T_SMEM_BYTES = T_OFF_SMALL + sizeof(Small);
static_assert(T_SMEM_BYTES <= 227 * 1024 && T_OFF_QT % 1024 == 0 && T_OFF_WT % 1024 == 0, "Toeplitz layout");
// Tensor memory (Toeplitz layout): K words at 0 (a dimension a column; one buffer); score
// accumulators of buffer b at 128 + 64 b, four of them 16 columns apart (n = 8 g + k); the four
// P.V accumulators at 256 + 32 a (n = 16 g + k); V words at 384 (a key a column, channel c in
// lane c). Each MMA group (16 K steps of 8 elements x 4 bytes) is issued by four threads, four
// consecutive K steps each into an accumulator of its own: a tcgen05.mma costs its issuing
// thread tens of cycles, and separate issuers overlap.
constexpr uint32_t T_COL_S = 128, T_COL_O = 256, T_COL_V = 384;
constexpr uint32_t V_BIAS = 1u << 30;  // (the K bias is 2^W, W the launch's window bits)
static_assert(OFF_V % 1024 == 0 && OFF_Q % 16 == 0 && OFF_W % 16 == 0 && OFF_RAWV % 1024 == 0, "operand alignment");
// K fetch modes: 0 dense bulk copies of contiguous runs; 1 RANGE through the tensor map (one box
// of 128 rows per half); 2 PAGED through the tensor map (boxes of `kbox` rows, a page or a
// 128-row part of one; tiles start on page boundaries)
constexpr int KM_DENSE = 0, KM_RANGE = 1, KM_PAGED = 2;

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

// One warp: bulk copies of keys [j0, j0 + n) of V (128 bf16 per row) into the dense raw tile
// `raw`; lane 0 arms the barrier. RANGE: one contiguous run from `kvbase` (the segment's kv_base,
// read once per CTA). PAGED: one run per page touched, run r issued by lane r % 32, each lane
// reading its own page-table entry (or taking it from page_pref, read ahead), so the lookups
// overlap instead of chaining.
__device__ __forceinline__ void fetch_rows(const Prob& P, const uint16_t* src, int32_t row0, int64_t kvbase,
                                           int64_t j0, int n, uint8_t* raw, uint64_t* bar, int64_t page_pref = -1) {
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

// The page-table entry of box `lane` of the K tile at j0 (KM_PAGED; -1 when the box lies past kend)
__device__ __forceinline__ int64_t kbox_page(const Prob& P, int32_t row0, int64_t j0, int64_t kend, int kbox) {
  const int64_t j = j0 + (int64_t)(threadIdx.x & 31) * kbox;
  if (j >= kend || j >= j0 + BK) return -1;
  return (int64_t)P.page_table[(int64_t)(row0 / P.hq) * P.max_pages + j / P.page_size];
}

// One warp: the K rows of keys [j0, j0 + n) into raw tile `raw`; lane 0 arms the barrier.
// KM_RANGE / KM_PAGED: 2D tensor-map boxes into the two swizzled halves (a box's rows land at its
// tile rows, so each 8-row group starts on a 1024-byte boundary); `pref`: kbox_page of this
// lane's box. KM_DENSE: contiguous runs into 256-byte rows (fetch_rows; `pref` its page_ahead).
__device__ __forceinline__ void fetch_k(const Prob& P, const CUtensorMap* tm, int kmode, int kbox, int32_t row0,
                                        int64_t kvbase, int64_t j0, int n, uint8_t* raw, uint64_t* bar, int64_t pref) {
  const int lane = threadIdx.x & 31;
  if (kmode == KM_RANGE) {
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(bar, 2u * KHALF);
      const int y = (int)(kvbase + j0);
      tc::tma_load_2d(raw, tm, 0, y, bar);
      tc::tma_load_2d(raw + KHALF, tm, 64, y, bar);
    }
    return;
  }
  if (kmode == KM_PAGED) {
    const int nbox = (n + kbox - 1) / kbox;
    if (lane == 0) tc::mbar_arrive_expect_tx(bar, (uint32_t)nbox * 2u * (uint32_t)kbox * 128u);
    __syncwarp();
    if (lane < nbox) {
      const int64_t b = row0 / P.hq;
      const int kvh = (int)(row0 - b * P.hq) / P.group;
      const int64_t j = j0 + (int64_t)lane * kbox;
      const int y = (int)((pref * P.hkv + kvh) * P.page_size + j % P.page_size);
      tc::tma_load_2d(raw + lane * kbox * 128, tm, 0, y, bar);
      tc::tma_load_2d(raw + KHALF + lane * kbox * 128, tm, 64, y, bar);
    }
    return;
  }
  fetch_rows(P, P.k, row0, kvbase, j0, n, raw, bar, pref);
}

// Named barrier over `n` threads with an AND / OR vote.
__device__ __forceinline__ bool group_sync_and(int id, int n, bool p) {
  int r;
  asm volatile(
      "{\n\t.reg .pred q, rr;\n\t"
      "setp.ne.s32 q, %1, 0;\n\t"
      "bar.red.and.pred rr, %2, %3, q;\n\t"
      "selp.s32 %0, 1, 0, rr;\n\t}\n"
      : "=r"(r)
      : "r"((int)p), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool group_sync_or(int id, int n, bool p) {
  int r;
  asm volatile(
      "{\n\t.reg .pred q, rr;\n\t"
      "setp.ne.s32 q, %1, 0;\n\t"
      "bar.red.or.pred rr, %2, %3, q;\n\t"
      "selp.s32 %0, 1, 0, rr;\n\t}\n"
      : "=r"(r)
      : "r"((int)p), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void group_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// named barriers: 1 consumers (256 threads), 2 K producers (128), 3 V producers (128)
constexpr int BAR_C = 1, BAR_K = 2, BAR_V = 3;

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

// The part of bf16 `bits` (value v) that FLOORING v 2^-lsb to an integer dropped, v 2^-lsb -
// floor(v 2^-lsb) in [0, 1), in units 2^-24, itself floored (< 2^24); `lost2` when bits remain
// below that unit.
__device__ __forceinline__ int32_t lost_part24(uint32_t bits, int lsb, int& lost2) {
  int32_t m, e;
  decode_bf16(bits, m, e);
  lost2 = 0;
  const uint32_t mag = (uint32_t)(m < 0 ? -m : m);
  const int s = lsb - e;  // the bits of mag below the unit 2^lsb
  if (s <= 0 || mag == 0) return 0;
  const uint32_t low = s >= 32 ? mag : (mag & ((1u << s) - 1));  // units 2^e, < 2^9
  if (low == 0) return 0;
  // the dropped fraction is low / 2^s for v >= 0 and 1 - low / 2^s for v < 0
  if (s <= 24) return (int32_t)((m < 0 ? (1u << s) - low : low) << (24 - s));
  const int r = s - 24;
  if (m >= 0) {
    if (r >= 32) {
      lost2 = 1;
      return 0;
    }
    const uint32_t dx = low >> r;
    lost2 = (dx << r) != low;
    return (int32_t)dx;
  }
  // floor((2^s - low) / 2^r) = 2^24 - ceil(low / 2^r); a remainder iff low is not a multiple of 2^r
  lost2 = 1;
  if (r >= 32) return (1 << 24) - 1;
  const uint64_t rm = ((uint64_t)1 << r) - 1;
  lost2 = (low & rm) != 0;
  return (int32_t)((1u << 24) - (uint32_t)(((uint64_t)low + rm) >> r));
}

// Fixed point (fixq) of the four bf16 of words w0, w1 at lsb, out of line: only keys whose
// largest element lies below 2^-100 take it, and inlined its 32 copies would crowd the K
// producers' hot loop
static __device__ __noinline__ uint4 fixq4_ool(uint32_t w0, uint32_t w1, int lsb) {
  int lost = 0, b2 = 0;
  uint4 r;
  r.x = (uint32_t)fixq(w0 & 0xFFFFu, lsb, lost, b2);
  r.y = (uint32_t)fixq(w0 >> 16, lsb, lost, b2);
  r.z = (uint32_t)fixq(w1 & 0xFFFFu, lsb, lost, b2);
  r.w = (uint32_t)fixq(w1 >> 16, lsb, lost, b2);
  return r;
}

// logit_interval_f64 out of line (pairs with lossy elements only): bits 0-31 the logit, bit 32
// `differ`, bit 33 `done`
static __device__ __noinline__ uint64_t logit_interval_ool(int64_t acc, uint64_t err, int sexp, double am_d, int32_t ae) {
  uint32_t fb = 0;
  bool differ = false;
  const bool done = f64::logit_interval_f64(acc, err, sexp, am_d, ae, fb, differ);
  return (uint64_t)fb | ((uint64_t)differ << 32) | ((uint64_t)done << 33);
}

// The logit of a score whose windows lost bits, from the exact binary64 correction of its lossy
// elements (Toeplitz layout; out of line, the pairs with lost bits only): with q = Q 2^qlsb + dq and
// k = K 2^klsb + dk, q k - Q K 2^(qlsb + klsb) = Q 2^qlsb dk + dq k summed over the row's lossy
// dimensions (k exact from K and dk) and the key's other lossy elements; one rounding per term
// and per sum, |corr - c| <= (n + 2) 2^-53 sum |terms|. Bits 0-31 the logit, bit 32 set when it
// is certified; 0 when a list is incomplete (the caller falls back on the truncation bound).
static __device__ __noinline__ uint64_t lossy_corr_logit(const Small& S, const KcArea& KC, const int32_t* qfx_g, int g,
                                                         int b, int key, bool klossy, int64_t acc, int qlsb, int klsb,
                                                         double am_d, int32_t ae) {
  const int nql = S.nqlk;
  const int n0 = klossy ? KC.kcn[b][0][key] : 0, n1 = klossy ? KC.kcn[b][1][key] : 0;
  if (nql < 0 || n0 > 2 || n1 > 2 || qlsb < -1000 || klsb < -1000 || qlsb > 1000 || klsb > 1000) return 0;
  const double pq = __hiloint2double((qlsb + 1023) << 20, 0), pk = __hiloint2double((klsb + 1023) << 20, 0);
  double c = 0.0, a = 0.0;
  int cnt = 0;
  for (int n = 0; n < nql; ++n) {  // the row's lossy dimensions
    const int i = S.qlk[n];
    if (!((S.qlossy[g][i >> 5] >> (i & 31)) & 1u)) continue;
    double dk = 0.0;
    for (int h = 0; h < 2; ++h)
      for (int e = 0; e < (h ? n1 : n0); ++e)
        if (KC.kci[b][h][key][e] == i) dk = (double)KC.kcd[b][h][key][e];
    const double k = (double)S.kqv[b][key][n] * pk + dk;  // the element itself, exact
    const double Qs = dk != 0.0 ? (double)qfx_g[i] * pq : 0.0;
    const double t = __fma_rn(Qs, dk, (double)KC.qdq[g][n] * k);
    c += t;
    a += fabs(t);
    ++cnt;
  }
  for (int h = 0; h < 2; ++h)  // the key's other lossy elements: Q 2^qlsb dk, exact
    for (int e = 0; e < (h ? n1 : n0); ++e) {
      const int i = KC.kci[b][h][key][e];
      if ((S.qlossy[g][i >> 5] >> (i & 31)) & 1u) continue;
      const double t = (double)qfx_g[i] * pq * (double)KC.kcd[b][h][key][e];
      c += t;
      a += fabs(t);
      ++cnt;
    }
  const double err = (double)(cnt + 2) * 1.1102230246251565e-16 * a * 1.000001;
  uint32_t fb = 0;
  if (!f64::logit_f64_corr(acc, qlsb + klsb, c, err, am_d, ae, fb)) return 0;
  return (uint64_t)fb | (1ull << 32);
}

// q row g's fixed-point element i from its balanced digit planes in the score B tile
__device__ __forceinline__ int32_t q_fix(const uint8_t* sQ, int g, int i) {
  int32_t x = 0;
#pragma unroll
  for (int t = NQ - 1; t >= 0; --t) x = x * 256 + (int32_t)(int8_t)sQ[tc::kmajor_off(4 * g + t, i, NSQ)];
  return x;
}

// bytes 0, 1, 2 of four words as three words (byte k of word j -> byte j of output k)
__device__ __forceinline__ void transpose3(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, uint32_t& p0,
                                           uint32_t& p1, uint32_t& p2) {
  const uint32_t a = __byte_perm(x0, x1, 0x5140), c = __byte_perm(x2, x3, 0x5140);
  const uint32_t b = __byte_perm(x0, x1, 0x7362), d = __byte_perm(x2, x3, 0x7362);
  p0 = __byte_perm(a, c, 0x5410);
  p1 = __byte_perm(a, c, 0x7632);
  p2 = __byte_perm(b, d, 0x5410);
}

// RPT: row slots per consumer thread (rows h, h + NWG, ..): segments of at most NWG RPT rows.
// NC: consumer warps (8: two warpgroups, rows split between them; 4: one warpgroup with every row).
// KW: K producer warps (4: one thread a key; 8: two threads a key, each half the dimensions).
// With 8 consumer and 8 K warps the block has 640 threads and rebalances registers per role
// (setmaxnreg): the launch gives 96 a thread, the producers drop to REG_PRODUCER and the consumers
// rise to REG_CONSUMER (256 x 120 + 384 x 80 = 61,440 = 640 x 96).
// SCA (Toeplitz layout): score accumulators, one issuer each (16 / SCA K steps an issuer): fewer
// accumulators mean fewer TMEM reads and adds for the consumers, more MMAs an issuing K producer.
template <int RPT, int NC, int KW, int SCA = 4>
__global__ void __launch_bounds__(threads_of<NC, KW>(), 1)
    tc_decode_kernel(Prob P, const int32_t* __restrict__ seg_rows, const __grid_constant__ CUtensorMap tmk, int kmode,
                     int kbox) {
  constexpr int THREADS = threads_of<NC, KW>();
  constexpr bool REBAL = THREADS > 512;  // per-role registers
  static_assert(!REBAL || (NC == 8 && KW == 8 && REG_SPLIT <= THREADS * REG_LAUNCH), "register split");
  constexpr int NWG = NC / 4;          // consumer warpgroups
  constexpr int KW0 = NC;              // first K producer warp
  constexpr int VW0 = NC + KW;         // first V producer warp
  constexpr int KWN = KW;              // K producer warps: 4 or 8
  constexpr int KH = KWN / 4;          // K threads a key (each takes D / KH dimensions)
  constexpr int BLKS = 4 / KH;         // 32-dimension blocks a K thread slices
  // One row slot (segments of <= 2 rows): the K digits and the score accumulators are double-
  // buffered in tensor memory, so the K producers run up to two tiles ahead of the consumers'
  // pass 1 instead of one. Tile i uses score buffer sbuf(i) and that buffer's barrier phase
  // spar(i).
  constexpr bool DB = RPT == 1;
  // the 640-thread instantiation uses the Toeplitz layout (K and V words in tensor memory)
  constexpr bool TOEP = REBAL;
  constexpr int VST = TOEP ? 3 : 2;  // raw V staging buffers
  static_assert(!TOEP || DB, "Toeplitz layout: segments of at most two rows");
  constexpr uint32_t SPL = DB ? 8u : 32u;  // score accumulator columns a key digit plane
  constexpr uint32_t COLO = TOEP ? T_COL_O : DB ? DB_COL_O : COL_O;
  auto sbuf = [](int i) { return DB ? (i & 1) : 0; };
  auto spar = [](int i) { return (uint32_t)(DB ? (i >> 1) & 1 : i & 1); };
  auto col_k = [](int b) { return TOEP ? 0u : DB ? 128u * (uint32_t)b : COL_K; };
  auto col_s = [](int b) { return TOEP ? T_COL_S + 64u * (uint32_t)b : DB ? DB_COL_S + 32u * (uint32_t)b : COL_S; };
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* rawk = smem + OFF_RAWK;
  uint8_t* rawv = smem + OFF_RAWV;
  uint8_t* sV = smem + OFF_V;  // (not in the Toeplitz layout)
  uint8_t* sQ = smem + (TOEP ? T_OFF_QT : OFF_Q);
  uint8_t* sW = smem + (TOEP ? T_OFF_WT : OFF_W);
  uint32_t* sT = (uint32_t*)(smem + (TOEP ? T_OFF_T : OFF_T));
  int32_t* qfx = (int32_t*)(smem + T_OFF_QF);    // Toeplitz: the rows' fixed-point query elements
  uint64_t* wval = (uint64_t*)(smem + T_OFF_WV);  // Toeplitz: the tile's weights W[g][key]
  Small& S = *(Small*)(smem + (TOEP ? T_OFF_SMALL : OFF_SMALL));
  EA_PT_DECL

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seg = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
  // the swizzled tensor-map boxes land on 1024-byte boundaries of the shared window
  if (tc::smem_u32(smem) & 1023u) kmode = KM_DENSE;

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
  if (TOEP)  // both B tiles start zero (the unused digit positions and rows stay zero)
    for (int i = tid; i < (int)((T_QROWS + T_WROWS) * T_KB / 16); i += THREADS) ((uint4*)sQ)[i] = make_uint4(0, 0, 0, 0);
  if (tid < 256) S.td[tid] = f64::g_exp2_d64[tid];
  if (tid == 0) {
    tc::mbar_init(&S.bar_rk[0], 1);
    tc::mbar_init(&S.bar_rk[1], 1);
    tc::mbar_init(&S.bar_rv[0], 1);
    tc::mbar_init(&S.bar_rv[1], 1);
    tc::mbar_init(&S.bar_rv[2], 1);
    // one commit per issuer (a key / value digit, or in the Toeplitz layout four K steps)
    tc::mbar_init(&S.bar_smma[0], TOEP ? SCA : NK);
    tc::mbar_init(&S.bar_smma[1], TOEP ? SCA : NK);
    tc::mbar_init(&S.bar_pv, NV);
    tc::mbar_init(&S.bar_p1[0], 1);
    tc::mbar_init(&S.bar_p1[1], 1);
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
  if (nrows > NWG * RPT || (TOEP && (tc::smem_u32(smem) & 1023u))) {
    // more rows than this instantiation keeps sums for, or swizzled tiles off their 1024-byte
    // alignment (a launch error): every row of the segment goes to the exact tier, and the run
    // is flagged
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
  // split s covers keys [kbeg, kend): cut points rounded down to whole 128-key tiles, so tiles of
  // a paged sequence start on page boundaries (any split layout gives the same bits)
  const int64_t kbeg = (maxlen * split / nsplit) & ~(int64_t)(BK - 1);
  const int64_t kend = split + 1 == nsplit ? maxlen : ((maxlen * (split + 1) / nsplit) & ~(int64_t)(BK - 1));
  const int ntiles = (int)((kend - kbeg + BK - 1) / BK);
  const int64_t kvbase = P.kind == MASK_RANGE ? P.kv_base[row0] : 0;
  // MMA N sizes for this segment's rows (4 query digits and 6 weight digits a row)
  const int nsq = nrows <= 2 ? 8 : nrows <= 4 ? 16 : 32;
  const int npv = nrows <= 2 ? 16 : nrows <= 4 ? 32 : 48;
  if (warp == 0) tc::tmem_alloc(&S.tmem, TMEM_COLS);
  // the first two tiles' K (warp 11) and V (warp 15) fetches
  if (warp == VW0 - 1)
    for (int t = 0; t < 2 && t < ntiles; ++t) {
      const int64_t j0 = kbeg + (int64_t)t * BK;
      const int64_t pref = kmode == KM_PAGED ? kbox_page(P, row0, j0, kend, kbox) : page_ahead(P, row0, j0, kend);
      fetch_k(P, &tmk, kmode, kbox, row0, kvbase, j0, (int)min((int64_t)BK, kend - j0), rawk + t * RAWK_BUF,
              &S.bar_rk[t], pref);
    }
  if (warp == VW0 + 3)
    for (int t = 0; t < VST && t < ntiles; ++t) {
      const int64_t j0 = kbeg + (int64_t)t * BK;
      fetch_rows(P, P.v, row0, kvbase, j0, (int)min((int64_t)BK, kend - j0), rawv + t * RAWV_BUF, &S.bar_rv[t]);
    }

  // ---------------- query rows -> balanced digit planes (warp g: row g) ----------------
  if (TOEP ? warp < 2 : warp < GD) {
    const int g = warp;
    int64_t qs = 0;  // the row's fixed-point sum (Toeplitz)
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
      uint32_t dq = 0;  // the four digits as bytes
#pragma unroll
      for (int s = 0; s < NQ; ++s) {
        const int32_t dg = s == NQ - 1 ? y : (int32_t)(int8_t)(y & 0xFF);
        if (TOEP) dq |= (uint32_t)(uint8_t)(int8_t)dg << (8 * s);
        else sQ[tc::kmajor_off(4 * g + s, i, NSQ)] = (uint8_t)(int8_t)dg;
        y = (y - dg) >> 8;
      }
      if (TOEP) {
        // score B row (g, k), bytes 4 i .. 4 i + 3: digits Q_k, Q_(k-1), Q_(k-2), Q_(k-3) (zero
        // outside 0..3)
        const uint32_t sel[7] = {0x4440u, 0x4401u, 0x4012u, 0x0123u, 0x1234u, 0x2344u, 0x3444u};
#pragma unroll
        for (int k = 0; k < 7; ++k)
          *(uint32_t*)(sQ + tc::sw128_off(8 * g + k, 4 * i, T_QROWS)) = __byte_perm(dq, 0u, sel[k]);
        qfx[g * D + i] = x;
        qs += x;
      }
    }
    if (TOEP) {
#pragma unroll
      for (int o = 16; o; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    }
    if (lane == 0) {
      if (TOEP) S.qsum[g] = qs;
      S.qlsb[g] = lsb;
      if (bad && row >= 0) S.rst[g] = ST_DOMAIN;
    }
  }
  __syncthreads();
  if (tid == 0) {  // the dimensions where some query row lost bits (usually none)
    int n = 0;
    for (int wd = 0; wd < 4; ++wd) {
      uint32_t u = 0;
      for (int g = 0; g < nrows; ++g) u |= S.qlossy[g][wd];
      for (; u; u &= u - 1) {
        if (n < NQL) S.qlk[n] = 32 * wd + __ffs(u) - 1;
        ++n;
      }
    }
    S.nqlk = n <= NQL ? n : -1;
    if (TOEP && n <= NQL) {  // the rows' lost parts at the listed dimensions (exact, as dk)
      KcArea& KC = *(KcArea*)(smem + T_OFF_KC);
      for (int g = 0; g < 2; ++g)
        for (int m = 0; m < NQL; ++m) {
          float dq = 0.0f;
          if (g < nrows && m < n && S.rows[g] >= 0) {
            const int i = S.qlk[m];
            if ((S.qlossy[g][i >> 5] >> (i & 31)) & 1u) {
              const uint32_t qb = P.q[(int64_t)S.rows[g] * D + i];
              dq = (float)((double)__uint_as_float(qb << 16) -
                           (double)qfx[g * D + i] * __hiloint2double((max(S.qlsb[g], -1022) + 1023) << 20, 0));
            }
          }
          KC.qdq[g][m] = dq;
        }
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
  // consumer state (rows h, h + NWG, .. of channel c), live until the partials are written
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
  // floors of the tiles' shifts into N not yet added to Nerr (folded in before any rescale and at
  // the end, which gives Nerr's exact sequence of values where it is used)
  uint32_t nfl[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    R[i] = R_EMPTY;
    Tlo[i] = INT32_MAX;
    Z[i] = 0;
    N[i] = 0;
    Zerr[i] = 0;
    Nerr[i] = 0;
    nfl[i] = 0;
  }
  int32_t vec = INT32_MIN;  // this channel's VE as last applied to N

  if (warp >= KW0 && warp < VW0) {
    // ======================= K producers: one key per thread, digits into TMEM =======================
    if (REBAL) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_PRODUCER));
    const int kw = warp - KW0;
    const int khf = kw >> 2;  // which D / KH dimensions of the key this thread takes
    const int key = 32 * (warp & 3) + lane;
    const int nqlk = max(S.nqlk, 0);
    const uint32_t kbias = 1u << P.W;  // Toeplitz: key words x + 2^W (|x| < 2^W)
    const uint32_t tq = tmem + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's TMEM lane quadrant
    int waited = 0, issued = min(ntiles, 2);  // tiles [waited, issued) have fetches in flight
    bool mma_pend = false;
    int mma_last = 0;  // the last tile whose score MMAs this role issued
    // byte offset of 16-byte chunk c (dims 8c .. 8c + 7) of this thread's raw row: in the swizzled
    // halves (c / 8) * KHALF + 128 key + ((c % 8) ^ (key % 8)) 16, in dense rows 256 key + 16 c
    const bool swz = kmode != KM_DENSE;
    const uint32_t rbase = swz ? (uint32_t)key * 128u : (uint32_t)key * 256u;
    const uint32_t hstep = swz ? KHALF : 128u;
    const uint32_t x7 = swz ? (uint32_t)(key & 7) : 0u;
    int64_t kpref = -1;
    EA_PTK_INIT
    for (int i = 0; i < ntiles; ++i) {
      const int b = i & 1;
      const int64_t j0 = kbeg + (int64_t)i * BK;
      const int nvalid = (int)min((int64_t)BK, kend - j0);
      bool okw = tc::mbar_wait(&S.bar_rk[b], (uint32_t)(i >> 1) & 1u, P.wait_debug);
      if (!group_sync_and(BAR_K, KWN * 32, okw && !*(volatile int*)&S.abort)) {
        ok_wait = false;
        break;
      }
      waited = i + 1;
      // page-table entries of tile i + 2, read now for its fetch below
      if (warp == VW0 - 1 && i + 2 < ntiles)
        kpref = kmode == KM_PAGED ? kbox_page(P, row0, j0 + 2 * BK, kend, kbox) : page_ahead(P, row0, j0 + 2 * BK, kend);
      EA_PTK(0)
      const uint8_t* rawb = rawk + b * RAWK_BUF + rbase;
#define KCHUNK(c) (rawb + ((c) >> 3) * hstep + ((((uint32_t)(c) & 7u) ^ x7) << 4))
      const bool valid = key < nvalid;
      // pass A: the key's largest magnitude and its smallest nonzero one (two chains)
      uint32_t mx0 = 0, mx1 = 0, mk0 = NZ_NONE, mk1 = NZ_NONE;
      if (valid) {
#pragma unroll
        for (int cc = khf * (16 / KH); cc < (khf + 1) * (16 / KH); ++cc) {
          const uint4 a = *(const uint4*)KCHUNK(cc);
          const uint32_t m0 = a.x & 0x7FFF7FFFu, m1 = a.y & 0x7FFF7FFFu;
          const uint32_t m2 = a.z & 0x7FFF7FFFu, m3 = a.w & 0x7FFF7FFFu;
          mx0 = __vmaxu2(mx0, __vmaxu2(m0, m1));
          mx1 = __vmaxu2(mx1, __vmaxu2(m2, m3));
          mk0 = __vmins2(mk0, __vmins2(nz_key(m0), nz_key(m1)));
          mk1 = __vmins2(mk1, __vmins2(nz_key(m2), nz_key(m3)));
        }
      }
      uint32_t mx = __vmaxu2(mx0, mx1);
      mx = max(mx & 0xFFFFu, mx >> 16);
      int32_t mn = nz_key_min(__vmins2(mk0, mk1));
      if (KH == 2) {  // the other half of the key, from its other thread
        S.kscan[khf][key][0] = mx;
        S.kscan[khf][key][1] = (uint32_t)mn;
        group_sync(BAR_K, KWN * 32);
        mx = max(mx, S.kscan[khf ^ 1][key][0]);
        mn = min(mn, (int32_t)S.kscan[khf ^ 1][key][1]);
      }
      const int bad = mx >= 0x7F80u;
      const int lead = (mx == 0 || bad) ? INT32_MIN : lead_of_bits(mx);
      const int lsb = lead == INT32_MIN ? 0 : lead + 1 - P.W;
      const int ebase = lsb + 134;  // an element with exponent field E >= ebase loses no bits
      const bool fast = lead == INT32_MIN || (lsb >= -126 && lsb <= 126 &&
                                              (mn == 32767 || nz_key_mag(mn) >= ((uint32_t)ebase << 7)));
      const float sc = scale_of(max(-126, min(126, lsb)));
      // one K buffer: the score MMAs of tile i - 1 are done reading the K digits in tensor
      // memory; two score buffers: the consumers' pass 1 of tile i - 2 is done (so are its score
      // MMAs, and its score accumulators and key metadata slot are free)
      if (i > 0 && (!DB || TOEP || i >= 2)) {
        okw = true;
        if (DB && i >= 2) okw = tc::mbar_wait(&S.bar_p1[b], spar(i - 2), P.wait_debug);
        if (!DB || TOEP) okw = okw && tc::mbar_wait(&S.bar_smma[sbuf(i - 1)], spar(i - 1), P.wait_debug);
        if (!group_sync_and(BAR_K, KWN * 32, okw)) {
          ok_wait = false;
          break;
        }
        if (!DB) mma_pend = false;
      }
      tc::fence_after_sync();
      EA_PTK(1)
      // pass B: digits of 32 dims at a time (4 planes x 8 columns), stored to this key's TMEM lane.
      // x = trunc(k 2^-lsb) through fp32 is exact for every finite element when lsb lies in
      // [-126, 126] (the product is exact or below 1); a key whose largest element is below
      // 2^-100 (lsb < -126) takes the integer conversion.
      const bool norm = lead == INT32_MIN || lsb >= -126;
#pragma unroll 1
      for (int blk = khf * BLKS; blk < (khf + 1) * BLKS; ++blk) {
        uint32_t pl[NK][8];
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          uint4 a = make_uint4(0u, 0u, 0u, 0u);
          if (valid && lead != INT32_MIN) a = *(const uint4*)KCHUNK(4 * blk + g4);
          const uint32_t w[4] = {a.x, a.y, a.z, a.w};
          uint32_t xs[8];
          if (norm) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              xs[2 * q] = fixf_lo(w[q], sc);
              xs[2 * q + 1] = fixf_hi(w[q], sc);
            }
          } else {
            const uint4 lo = fixq4_ool(w[0], w[1], lsb), hi = fixq4_ool(w[2], w[3], lsb);
            xs[0] = lo.x, xs[1] = lo.y, xs[2] = lo.z, xs[3] = lo.w;
            xs[4] = hi.x, xs[5] = hi.y, xs[6] = hi.z, xs[7] = hi.w;
          }
          if (TOEP) {  // the words x + 2^W of dimensions 8 (4 blk + g4) .. + 7, one a column
#pragma unroll
            for (int e = 0; e < 8; ++e) xs[e] += kbias;
            tc::tmem_st8(tq + col_k(b) + 8 * (4 * blk + g4), xs);
          } else {
            transpose4(xs[0], xs[1], xs[2], xs[3], pl[0][2 * g4], pl[1][2 * g4], pl[2][2 * g4], pl[3][2 * g4]);
            transpose4(xs[4], xs[5], xs[6], xs[7], pl[0][2 * g4 + 1], pl[1][2 * g4 + 1], pl[2][2 * g4 + 1],
                       pl[3][2 * g4 + 1]);
          }
        }
        if (!TOEP) {
#pragma unroll
          for (int t = 0; t < NK; ++t) tc::tmem_st8(tq + col_k(b) + 32 * t + 8 * blk, pl[t]);
        }
      }
      // the elements that lost bits (exponent field below ebase), for the consumers' error bound
      uint32_t lmk[4] = {0u, 0u, 0u, 0u};
      if (!fast && valid) {
        const uint32_t thr = (uint32_t)max(ebase, 0) << 7;
        int nkc = 0;  // Toeplitz: this half's lossy elements, the first two with their lost parts
#pragma unroll 1
        for (int cc = khf * (16 / KH); cc < (khf + 1) * (16 / KH); ++cc) {
          const uint4 a = *(const uint4*)KCHUNK(cc);
          const uint32_t w[4] = {a.x, a.y, a.z, a.w};
          uint32_t bits = 0;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t mg = (w[e >> 1] >> (16 * (e & 1))) & 0x7FFFu;
            bits |= (uint32_t)(mg != 0 && mg < thr) << e;
          }
          lmk[cc >> 2] |= bits << (8 * (cc & 3));
          if (TOEP) {
            KcArea& KC = *(KcArea*)(smem + T_OFF_KC);
            for (uint32_t m = bits; m; m &= m - 1) {
              const int e = __ffs(m) - 1;
              if (nkc < 2) {
                const uint32_t bb = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
                int lost = 0, b2 = 0;
                const int32_t x = fixq(bb, lsb, lost, b2);
                // k - K 2^lsb: the bits of k below the window, exact in binary64 and in fp32
                const double dk = (double)__uint_as_float(bb << 16) -
                                  (double)x * __hiloint2double((max(lsb, -1022) + 1023) << 20, 0);
                KC.kci[b][khf][key][nkc] = (uint8_t)(8 * cc + e);
                KC.kcd[b][khf][key][nkc] = (float)dk;
              }
              ++nkc;
            }
          }
        }
        if (TOEP) ((KcArea*)(smem + T_OFF_KC))->kcn[b][khf][key] = (uint8_t)min(nkc, 255);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (q / (4 / KH) == khf) S.klossy[b][key][q] = lmk[q];
      if (khf == 0) {
        S.klsb[b][key] = (int16_t)lsb;
        S.kbad[b][key] = (uint8_t)(valid && bad);
      }
      // the key's fixed-point values where some query row is lossy (the consumers' error bound)
      for (int n = 0; n < nqlk; ++n) {
        int lost = 0, b2 = 0;
        const int ii = S.qlk[n];
        if (ii / (D / KH) != khf) continue;
        const uint32_t kb = valid ? *(const uint16_t*)(KCHUNK(ii >> 3) + 2 * (ii & 7)) : 0u;
        S.kqv[b][key][n] = lead == INT32_MIN ? 0 : fixq(kb, lsb, lost, b2);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      EA_PTK(2)
      // every K thread is done with the raw rows of tile i: fetch tile i + 2 into them
      group_sync(BAR_K, KWN * 32);
      if (i + 2 < ntiles) {
        if (warp == VW0 - 1)
          fetch_k(P, &tmk, kmode, kbox, row0, kvbase, j0 + 2 * BK, (int)min((int64_t)BK, kend - j0 - 2 * BK),
                  rawk + b * RAWK_BUF, &S.bar_rk[b], kpref);
        issued = i + 3;
      }
      // one buffer: the consumers are done with the score accumulators of tile i - 1
      if (!DB) {
        okw = i > 0 ? tc::mbar_wait(&S.bar_p1[0], spar(i - 1), P.wait_debug) : true;
        if (!group_sync_and(BAR_K, KWN * 32, okw)) {
          ok_wait = false;
          break;
        }
      }
      EA_PTK(3)
      if (TOEP) {
        // score MMAs of tile i: lane 0 of K warp a < SCA issues K steps 16 a / SCA .. (dimensions
        // 128 a / SCA ..) into score accumulator a (N = 8 columns a row)
        if (lane == 0 && kw < SCA) {
          tc::fence_after_sync();
          const uint32_t idesc = tc::idesc_i8(128, 8 * nrows, false, true);
          const uint32_t qa = tc::smem_u32(sQ);
#pragma unroll
          for (int j = 0; j < 16 / SCA; ++j) {
            const int ks = (16 / SCA) * kw + j;
            tc::mma_i8_tmem_a(tmem + col_s(b) + 16 * kw, tmem + col_k(b) + 8 * ks,
                              tc::smem_desc_sw128(qa + (ks >> 2) * (T_QROWS / 8) * 1024 + (ks & 3) * 32, 1024), idesc,
                              j > 0);
          }
          tc::mma_commit(tc::smem_u32(&S.bar_smma[sbuf(i)]));
        }
      } else if (lane == 0 && kw < NK) {
        // score MMAs of tile i: key digit plane t (A in TMEM) by lane 0 of K warp t; an issuing
        // thread waits while the tensor core takes its operands, so four issuers share that wait
        const int t = kw;
        tc::fence_after_sync();
        constexpr uint32_t lbo_b = (NSQ / 8) * 128;
        const uint64_t bd0 = tc::smem_desc(tc::smem_u32(sQ), lbo_b, 128);
        const uint32_t idesc = tc::idesc_i8(128, nsq, t == NK - 1, true);
#pragma unroll
        for (int ks = 0; ks < D / 32; ++ks)
          tc::mma_i8_tmem_a(tmem + col_s(b) + SPL * t, tmem + col_k(b) + 32 * t + 8 * ks,
                            bd0 + ((ks * 2 * lbo_b) >> 4), idesc, ks > 0);
        tc::mma_commit(tc::smem_u32(&S.bar_smma[sbuf(i)]));
      }
      mma_pend = true;
      mma_last = i;
    }
#undef KCHUNK
    EA_PT_FLUSH_RANGE(256, 8, 12)
    if (!ok_wait) S.abort = 1;
    // what this role still has in flight gets a bounded wait before shared and tensor memory go
    for (int t = waited; t < issued; ++t) tc::mbar_wait(&S.bar_rk[t & 1], (uint32_t)(t >> 1) & 1u, P.wait_debug);
    // (each issuer's commit covers its earlier MMAs: the last tile's phase covers every tile)
    if (mma_pend) tc::mbar_wait(&S.bar_smma[sbuf(mma_last)], spar(mma_last), P.wait_debug);
  } else if (warp >= VW0 && warp < VW0 + 4) {
    // ======================= V producers: value digits into shared memory =======================
    if (REBAL) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_PRODUCER));
    const int vt = tid - VW0 * 32;
    const int cp = vt & 63, kh = vt >> 6;  // channels 2 cp, 2 cp + 1; keys 64 kh .. 64 kh + 63
    // Slot s of this thread holds channel 2 cp + (s ^ swp): a quarter warp's digit stores then
    // cover all 8 16-byte slots of a core matrix (no bank conflicts). The slot's value is taken out
    // of the 32-bit word of both channels by one byte permute (which also zeroes it for a channel
    // without digits).
    const int swp = (cp >> 2) & 1;
    int waited = 0, issued = min(ntiles, VST);  // tiles [waited, issued) have fetches in flight
    EA_PTV_INIT
    for (int i = 0; i < ntiles; ++i) {
      const int b = i % VST, par = i & 1;  // raw buffer; tile parity of the channel data
      const int64_t j0 = kbeg + (int64_t)i * BK;
      const int nvalid = (int)min((int64_t)BK, kend - j0);
      const int64_t pref = warp == VW0 + 3 ? page_ahead(P, row0, j0 + VST * BK, kend) : -1;
      bool okw = tc::mbar_wait(&S.bar_rv[b], (uint32_t)(i / VST) & 1u, P.wait_debug);
      if (!group_sync_and(BAR_V, 128, okw && !*(volatile int*)&S.abort)) {
        ok_wait = false;
        break;
      }
      waited = i + 1;
      EA_PTV(0)
      const uint8_t* vsrc = rawv + b * RAWV_BUF + (64 * kh) * (DV * 2) + cp * 4;  // key 64 kh + jj at jj * 256
      const int nv = min(64, max(0, nvalid - 64 * kh));  // this thread's valid keys
      // per channel (16-bit half) the largest magnitude and the key of the smallest nonzero one
      uint32_t mxw, mnw;
      {
        uint32_t x0 = 0, x1 = 0, x2 = 0, x3 = 0;
        uint32_t n0 = NZ_NONE, n1 = NZ_NONE, n2 = NZ_NONE, n3 = NZ_NONE;
        if (nv == 64) {  // full: no bounds test per load
#pragma unroll 4
          for (int jj = 0; jj < 64; jj += 4) {
            const uint32_t a0 = *(const uint32_t*)(vsrc + jj * (DV * 2)) & 0x7FFF7FFFu;
            const uint32_t a1 = *(const uint32_t*)(vsrc + (jj + 1) * (DV * 2)) & 0x7FFF7FFFu;
            const uint32_t a2 = *(const uint32_t*)(vsrc + (jj + 2) * (DV * 2)) & 0x7FFF7FFFu;
            const uint32_t a3 = *(const uint32_t*)(vsrc + (jj + 3) * (DV * 2)) & 0x7FFF7FFFu;
            x0 = __vmaxu2(x0, a0);
            x1 = __vmaxu2(x1, a1);
            x2 = __vmaxu2(x2, a2);
            x3 = __vmaxu2(x3, a3);
            n0 = __vmins2(n0, nz_key(a0));
            n1 = __vmins2(n1, nz_key(a1));
            n2 = __vmins2(n2, nz_key(a2));
            n3 = __vmins2(n3, nz_key(a3));
          }
        } else {
#pragma unroll 4
          for (int jj = 0; jj < nv; ++jj) {
            const uint32_t a0 = *(const uint32_t*)(vsrc + jj * (DV * 2)) & 0x7FFF7FFFu;
            x0 = __vmaxu2(x0, a0);
            n0 = __vmins2(n0, nz_key(a0));
          }
        }
        mxw = __vmaxu2(__vmaxu2(x0, x1), __vmaxu2(x2, x3));
        mnw = __vmins2(__vmins2(n0, n1), __vmins2(n2, n3));
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // physical channel 2 cp + h
        uint32_t m = (mxw >> (16 * h)) & 0xFFFFu;
        if (m >= 0x7F80u) {
          // a NaN / inf value: a domain error for the rows that see its key; the channel's range
          // comes from the finite values (the rows that do not see it use them)
          m = 0;
#pragma unroll 1
          for (int jj = 0; jj < nv; ++jj) {
            const uint32_t e = (*(const uint32_t*)(vsrc + jj * (DV * 2)) >> (16 * h)) & 0x7FFFu;
            if (e >= 0x7F80u) {
              for (int g = 0; g < nrows; ++g)
                if (S.rows[g] >= 0 && j0 + 64 * kh + jj < S.len[g]) atomicMax(&S.rst[g], ST_DOMAIN);
            } else {
              m = max(m, e);
            }
          }
        }
        S.ve4[kh][2 * cp + h] = (int16_t)(m == 0 ? INT16_MIN : lead_of_bits(m) + 1);
      }
      group_sync(BAR_V, 128);
      EA_PTV(1)
      // the P.V MMAs of tile i - 1 are done reading the value digits; the consumers, who issued
      // them after finishing tile i - 2, are also done with this parity's channel data
      if (i > 0) {
        okw = tc::mbar_wait(&S.bar_pv, (uint32_t)(i - 1) & 1u, P.wait_debug);
        if (!group_sync_and(BAR_V, 128, okw)) {
          ok_wait = false;
          break;
        }
      }
      EA_PTV(2)
      // running exponents of this thread's channels: the previous tiles' and this tile's
      int lsbh[2], keeph[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int ch = 2 * cp + h;
        int ve = S.ve[par ^ 1][ch];
        if (S.ve4[0][ch] != INT16_MIN) ve = max(ve, (int)S.ve4[0][ch]);
        if (S.ve4[1][ch] != INT16_MIN) ve = max(ve, (int)S.ve4[1][ch]);
        if (kh == 0) S.ve[par][ch] = ve;
        lsbh[h] = ve == INT32_MIN ? 0 : ve - FV;
        // a channel whose maximum lies at the very bottom of the bf16 range keeps no digits
        keeph[h] = (ve == INT32_MIN || lsbh[h] >= -126) ? 1 : 0;
      }
      S.vl_n[par][vt] = 0;
      group_sync(BAR_V, 128);  // this parity's lists reset, S.ve[par] complete
      // Values below the V window (an exponent field under lsb + 134): each goes to its channel's
      // correction list with the exact part the floor dropped, or past the list's capacity to the
      // bound; in a channel without digits every nonzero value is bounded.
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // physical channel 2 cp + h
        const int cc = 2 * cp + h;
        const int keep = keeph[h], lsb = lsbh[h];
        const uint32_t thr = keep ? ((uint32_t)max(lsb + 134, 0) << 7) : 0x8000u;  // all, when bounded
        const int32_t mk = (int32_t)(int16_t)((mnw >> (16 * h)) & 0xFFFFu);
        if (mk != 32767 && nz_key_mag(mk) < thr) {
          bool any = false;
#pragma unroll 1
          for (int jj = 0; jj < nv; ++jj) {
            const uint32_t bb = (*(const uint32_t*)(vsrc + jj * (DV * 2)) >> (16 * h)) & 0xFFFFu;
            const uint32_t mg = bb & 0x7FFFu;
            if (mg == 0 || mg >= thr) continue;
            any = true;
            if (!keep) continue;
            int lost2 = 0;
            const int32_t dx = lost_part24(bb, lsb, lost2);
            const uint32_t k = atomicAdd(&S.vl_n[par][cc], 1u);
            if (k < VLCAP) {
              S.vl_k[par][cc][k] = (uint16_t)((64 * kh + jj) | (lost2 << 8));
              S.vl_dx[par][cc][k] = dx;
            }
          }
          if (!keep && any) atomicAdd(&S.vl_n[par][cc], VL_BOUNDED);  // the whole channel is bounded
        }
      }
      if (TOEP) {
        // Words x + 2^30 of x = floor(v 2^-lsb) (|x| < 2^30): the product rounded toward -inf is
        // exact unless it is below 2^-126 in magnitude, where rounding down keeps the floor (0 or
        // -1); the conversion rounds down. A channel without digits (scale 0) counts its values
        // as 0. Keys past the tile's end keep whatever word their stale rows give: their weights
        // are 0 (and the digit-group bounds hold for any bytes). One channel a thread (its TMEM
        // lane), 8 keys a store.
        const int cv = 32 * (warp & 3) + lane;
        const int vev = S.ve[par][cv];
        const int lsbv = vev == INT32_MIN ? 0 : vev - FV;
        const float scv = (vev == INT32_MIN || lsbv >= -126) ? scale_of(lsbv) : 0.0f;
        const uint8_t* vcol = rawv + b * RAWV_BUF + 2 * cv;
        const uint32_t tv = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + T_COL_V;
        tc::fence_after_sync();  // after the P.V MMAs of tile i - 1 (the wait above)
#pragma unroll 2
        for (int j0 = 0; j0 < BK; j0 += 8) {
          uint32_t wv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t bits = *(const uint16_t*)(vcol + (j0 + e) * (DV * 2));
            const float y = __fmul_rd(__uint_as_float(bits << 16), scv);
            wv[e] = (uint32_t)__float2int_rd(y) + V_BIAS;
          }
          tc::tmem_st8(tv + j0, wv);
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
      } else {
        // per slot: the channel, the byte permute that places its bf16 in the high half of a zero
        // word (all zero without digits), and the scales of the two fused multiply-adds
        int chs[2];
        uint32_t sels[2];
        float schi[2], sclo[2], clampv[2];
  #pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          const int h = sl ^ swp;
          const int keep = h ? keeph[1] : keeph[0];
          const int l = keep ? (h ? lsbh[1] : lsbh[0]) : 0;
          chs[sl] = 2 * cp + h;
          sels[sl] = keep ? (h ? 0x3244u : 0x1044u) : 0x4444u;
          schi[sl] = scale_of(l + 8);       // 2^-(lsb + 8): the high part floor(x / 256)
          sclo[sl] = scale_of(l);           // 2^-lsb
          clampv[sl] = scale_of(-(l + 15));  // 2^(lsb + 15): above it x is a multiple of 256
        }
        // Digits of x = floor(v 2^-lsb) (|x| < 2^30) = 256 h + l: fmaf_rz(v, 2^-(lsb + 8), 1.5 2^23) is
        // 1.5 2^23 + h exactly (the product is exact, the sum positive, rounding toward zero is the
        // floor), whose low three bytes are h + 2^22; the same on v clamped to +-2^(lsb + 15) with
        // the scale 2^-lsb gives l = x mod 256 in the low byte (a value of magnitude 2^(lsb + 15) or
        // more is a multiple of 2^(lsb + 8), so l = 0 for it and for the clamp bound alike). The
        // digits are l and the three bytes of h + 2^22, i.e. of x + 2^30. Values of a channel
        // without digits count as 0. Sixteen keys per step, both slots from the same words.
  #pragma unroll 1
        for (int ck = 0; ck < 4; ++ck) {
          uint32_t w[16];
  #pragma unroll
          for (int jj = 0; jj < 16; ++jj) w[jj] = *(const uint32_t*)(vsrc + (16 * ck + jj) * (DV * 2));
  #pragma unroll
          for (int sl = 0; sl < 2; ++sl) {
            uint32_t pw[NV][4];
  #pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
              uint32_t fh[4], fl[4];
  #pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float f = __uint_as_float(__byte_perm(w[4 * c4 + e], 0u, sels[sl]));
                fh[e] = __float_as_uint(__fmaf_rz(f, schi[sl], V_MAGIC));
                fl[e] = __float_as_uint(__fmaf_rz(fminf(fmaxf(f, -clampv[sl]), clampv[sl]), sclo[sl], V_MAGIC));
              }
              transpose3(fh[0], fh[1], fh[2], fh[3], pw[1][c4], pw[2][c4], pw[3][c4]);
              pw[0][c4] = __byte_perm(__byte_perm(fl[0], fl[1], 0x0040), __byte_perm(fl[2], fl[3], 0x0040), 0x5410);
            }
  #pragma unroll
            for (int p = 0; p < NV; ++p)
              *(uint4*)(sV + p * V_PLANE + tc::kmajor_off(chs[sl], 64 * kh + 16 * ck, BK)) =
                  make_uint4(pw[p][0], pw[p][1], pw[p][2], pw[p][3]);
          }
        }
        tc::fence_async_smem();
      }
      group_sync(BAR_V, 128);
      EA_PTV(3)
      if (vt == 0) mbar_arrive(&S.bar_vready);  // value digits and channel data of tile i
      // the raw V rows of tile i are consumed: fetch tile i + VST into them
      if (i + VST < ntiles) {
        if (warp == VW0 + 3) {
          tc::fence_async_smem();
          fetch_rows(P, P.v, row0, kvbase, j0 + VST * BK, (int)min((int64_t)BK, kend - j0 - VST * BK),
                     rawv + b * RAWV_BUF, &S.bar_rv[b], pref);
        }
        issued = i + VST + 1;
      }
    }
    EA_PT_FLUSH_RANGE(VW0 * 32, 12, 16)
    if (!ok_wait) S.abort = 1;
    for (int t = waited; t < issued; ++t) tc::mbar_wait(&S.bar_rv[t % VST], (uint32_t)(t / VST) & 1u, P.wait_debug);
  } else {
    // ======================= consumer warpgroups: logits, weights, merges, drains =======================
    if (REBAL) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_CONSUMER));
    const uint32_t tlane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    int par = 0;
    bool pv_pending = false;
    uint32_t pv_ph = 0;
    EA_PT_INIT
    for (int i = 0; i < ntiles; ++i, par ^= 1) {
      const int64_t j0 = kbeg + (int64_t)i * BK;
      const int nvalid = (int)min((int64_t)BK, kend - j0);
      const uint32_t ph = (uint32_t)i & 1u;
      const int b = i & 1;
      {
        const bool okw = tc::mbar_wait(&S.bar_smma[sbuf(i)], spar(i), P.wait_debug);  // the score MMAs of tile i
        if (!group_sync_and(BAR_C, NC * 32, okw && !*(volatile int*)&S.abort)) {
          ok_wait = false;
          break;
        }
      }
      tc::fence_after_sync();
      EA_PT(0)
      // ---------------- pass 1: certified logits (lane: key; rows h, h + NWG, ..) ----------------
      bool unc = false;
      {
        const int key = c;
        const uint32_t* kl4 = S.klossy[b][key];
        const bool klossy = (kl4[0] | kl4[1] | kl4[2] | kl4[3]) != 0;
        const bool kbad = S.kbad[b][key];
        const int klsb = S.klsb[b][key];
        const int nqlk = S.nqlk;
#pragma unroll 1
        for (int g = h; g < nrows; g += NWG) {
          uint32_t dg[NK][4];
          uint32_t gt[8];  // Toeplitz: the digit groups G_0 .. G_6 of the biased key words
          if (TOEP) {  // the accumulators' digit groups, summed
            uint32_t g1[8];
            tc::tmem_ld8(tlane + col_s(b) + 8 * g, gt);
            tc::tmem_ld8(tlane + col_s(b) + 16 + 8 * g, g1);
            if (SCA == 4) {
              uint32_t g2[8], g3[8];
              tc::tmem_ld8(tlane + col_s(b) + 32 + 8 * g, g2);
              tc::tmem_ld8(tlane + col_s(b) + 48 + 8 * g, g3);
              tc::tmem_wait_ld();
#pragma unroll
              for (int k = 0; k < 7; ++k) gt[k] += g1[k] + g2[k] + g3[k];
            } else {
              tc::tmem_wait_ld();
#pragma unroll
              for (int k = 0; k < 7; ++k) gt[k] += g1[k];
            }
          } else {
#pragma unroll
            for (int t = 0; t < NK; ++t) tc::tmem_ld4(tlane + col_s(b) + SPL * t + 4 * g, dg[t]);
          }
          tc::tmem_wait_ld();
          uint32_t out = T_MASKED;
          if (key < nvalid && j0 + key < S.len[g] && S.rows[g] >= 0) {
            if (kbad) {
              atomicMax(&S.rst[g], ST_DOMAIN);
            } else {
              int64_t acc;
              if (TOEP) {
                // sum_k G_k 2^(8k) = q . (k + 2^W) exactly; taken mod 2^64, after the bias
                // 2^W q_sum is removed the result is q . k (|q . k| < 2^61)
                uint64_t u = 0;
#pragma unroll
                for (int k = 0; k < 7; ++k) u += (uint64_t)(int64_t)(int32_t)gt[k] << (8 * k);
                acc = (int64_t)(u - ((uint64_t)S.qsum[g] << P.W));
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
                acc = recomb<4>(lo4) + (int64_t)((uint64_t)recomb<3>(hi3) << 32);
              }
              const bool qlossy = (S.qlossy[g][0] | S.qlossy[g][1] | S.qlossy[g][2] | S.qlossy[g][3]) != 0;
              const int sexp = S.qlsb[g] + klsb;
              uint32_t fb;
              bool done = false, differ = false;
              uint64_t err = 0;
              if (TOEP && (qlossy || klossy)) {  // first the exact correction of the lost parts
                const uint64_t r = lossy_corr_logit(S, *(const KcArea*)(smem + T_OFF_KC), qfx + g * D, g, b, key, klossy,
                                                    acc, S.qlsb[g], klsb, am_d, P.ae);
                fb = (uint32_t)r;
                done = (r >> 32) & 1u;
              }
              if (done) {
              } else if (qlossy || klossy) {
                // |q k - Q K| <= |dq| |k| + |Q| |dk| over the lossy elements (units 2^(qlsb + klsb));
                // |k|'s fixed point as the K producers kept it (beyond their list: |K| < 2^W),
                // |Q| from the query digits
                if (nqlk >= 0) {
                  for (int n = 0; n < nqlk; ++n) {
                    const int ii = S.qlk[n];
                    if (!((S.qlossy[g][ii >> 5] >> (ii & 31)) & 1u)) continue;
                    const int32_t kf = S.kqv[b][key][n];
                    err += (uint64_t)(kf < 0 ? -kf : kf) + ((kl4[ii >> 5] >> (ii & 31)) & 1u);
                  }
                } else {
                  for (int wd = 0; wd < 4; ++wd) err += (uint64_t)__popc(S.qlossy[g][wd]) * ((1ull << P.W) + 1);
                }
                for (int wd = 0; wd < 4; ++wd) {
                  const uint32_t kl = kl4[wd];
                  for (uint32_t m = kl; m; m &= m - 1) {
                    const int ii = 32 * wd + __ffs(m) - 1;
                    const int32_t qf = TOEP ? qfx[g * D + ii] : q_fix(sQ, g, ii);
                    err += (uint64_t)(qf < 0 ? -qf : qf);
                  }
                }
                const uint64_t r = logit_interval_ool(acc, err, sexp, am_d, P.ae);
                fb = (uint32_t)r;
                differ = (r >> 32) & 1u;
                done = (r >> 33) & 1u;
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
                                                  : logit_exact_ool(acc, sexp, P.am, P.ae, t);
                if (ls == LOGIT_OK) out = rnd_to_f32_bits(t);
                else if (ls == LOGIT_UNCERTIFIED) out = T_UNCERT;
                else atomicMax(&S.rst[g], ST_DOMAIN);
              }
            }
          }
          sT[g * BK + key] = out;
          // tile bound of the certified logits: w = RN24(2^t) <= 2^(floor(t) + 1) < 2^(ceil(t) + 1);
          // a logit of magnitude 2^30 or more sends the row to the wide tier (whose exponents hold it)
          const float tf = __uint_as_float(out);
          int32_t rl = INT32_MIN, ll = INT32_MAX;
          if (out != T_MASKED && out != T_UNCERT) {
            if (fabsf(tf) < 1073741824.0f) {
              rl = __float2int_ru(tf) + 1;
              ll = __float2int_rd(tf);
            } else {
              atomicMax(&S.rst[g], ST_TIER3);
            }
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
      const bool any_unc = group_sync_or(BAR_C, NC * 32, unc);
      if (tid == 0) mbar_arrive(&S.bar_p1[sbuf(i)]);  // the score accumulators and key metadata of tile i are free
      EA_PT(1)
      // ---------------- exact scores of the uncertified pairs, one warp per pair ----------------
      if (any_unc) {
        for (int e0 = 0; e0 < nrows * BK; e0 += NC * 32) {
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
        group_sync(BAR_C, NC * 32);
        // the tile bounds again, now over the exact logits too
#pragma unroll 1
        for (int g = h; g < nrows; g += NWG) {
          const uint32_t tb = sT[g * BK + c];
          const float tf = __uint_as_float(tb);
          int32_t rl = INT32_MIN, ll = INT32_MAX;
          if (tb != T_MASKED) {
            if (fabsf(tf) < 1073741824.0f) {
              rl = __float2int_ru(tf) + 1;
              ll = __float2int_rd(tf);
            } else {
              atomicMax(&S.rst[g], ST_TIER3);  // |t| >= 2^30: the wide tier
            }
          }
          rl = __reduce_max_sync(0xffffffffu, rl);
          ll = __reduce_min_sync(0xffffffffu, ll);
          if (lane == 0) {
            S.rt[warp & 3][g] = rl;
            S.rtlo[warp & 3][g] = ll;
          }
        }
        group_sync(BAR_C, NC * 32);
      }
      EA_PT(2)
      // ---------------- pass 2: weights, W digits ----------------
#pragma unroll 1
      for (int g = h; g < nrows; g += NWG) {
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
            ws = weight_ool(t, Mi, Ei);
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
        if (TOEP) {
          // P.V B row (g, k), bytes 4 key .. 4 key + 3: weight digits W_k, W_(k-1), W_(k-2),
          // W_(k-3) (zero outside 0..5; W < 2^48)
          const uint32_t wl = (uint32_t)W, wh = (uint32_t)(W >> 32);
          const uint32_t sel[9] = {0x4440u, 0x4401u, 0x4012u, 0x0123u, 0x1234u, 0x2345u, 0x3456u, 0x4566u, 0x5666u};
#pragma unroll
          for (int k = 0; k < 9; ++k)
            *(uint32_t*)(sW + tc::sw128_off(16 * g + k, 4 * key, T_WROWS)) =
                k < 4 ? __byte_perm(wl, 0u, sel[k]) : __byte_perm(wl, wh, sel[k]);
          wval[g * BK + key] = W;
        } else {
#pragma unroll
          for (int wd = 0; wd < NW; ++wd) sW[tc::kmajor_off(6 * g + wd, key, NSW)] = (uint8_t)(W >> (8 * wd));
        }
        // the warp's weight sum from two 32-bit reductions of W's 24-bit halves (W < 2^48)
        const uint64_t zs = (uint64_t)__reduce_add_sync(0xffffffffu, (uint32_t)W & 0xFFFFFFu) +
                            ((uint64_t)__reduce_add_sync(0xffffffffu, (uint32_t)(W >> 24)) << 24);
        const uint32_t zl = __reduce_add_sync(0xffffffffu, lw);
        if (lane == 0) {
          S.zs[warp & 3][g] = zs;
          S.zl[warp & 3][g] = zl;
        }
      }
      tc::fence_async_smem();
      bool okw = tc::mbar_wait(&S.bar_vready, ph, P.wait_debug);  // the producers' value digits of tile i
      if (!group_sync_and(BAR_C, NC * 32, okw)) {
        ok_wait = false;
        break;
      }
      EA_PT(3)
      // ---------------- P.V MMAs: 4 value digits x (N: the rows' weight digits) ----------------
      if (TOEP) {
        // lane 0 of consumer warp a issues K steps 4 a .. 4 a + 3 (keys 32 a .. 32 a + 31; A: the
        // V words in tensor memory) into P.V accumulator a (N = 16 columns a row)
        if (lane == 0 && warp < NV) {
          tc::fence_after_sync();
          const uint32_t idesc = tc::idesc_i8(128, 16 * nrows, false, false);
          const uint32_t wa = tc::smem_u32(sW);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int ks = 4 * warp + j;
            tc::mma_i8_tmem_a(tmem + COLO + 32 * warp, tmem + T_COL_V + 8 * ks,
                              tc::smem_desc_sw128(wa + (ks >> 2) * (T_WROWS / 8) * 1024 + (ks & 3) * 32, 1024), idesc,
                              j > 0);
          }
          tc::mma_commit(tc::smem_u32(&S.bar_pv));
        }
      } else if (lane == 0 && warp < NV) {
        // value digit u to its own accumulator, issued by lane 0 of consumer warp u
        const int u = warp;
        tc::fence_after_sync();
        constexpr uint32_t lbo_a = (DV / 8) * 128, lbo_b = (NSW / 8) * 128;
        const uint64_t ad0 = tc::smem_desc(tc::smem_u32(sV + u * V_PLANE), lbo_a, 128);
        const uint64_t bd0 = tc::smem_desc(tc::smem_u32(sW), lbo_b, 128);
        const uint32_t idesc = tc::idesc_i8(128, npv, false, false);
#pragma unroll
        for (int ks = 0; ks < BK / 32; ++ks)
          tc::mma_i8(tmem + COLO + NSW * u, ad0 + ((ks * 2 * lbo_a) >> 4), bd0 + ((ks * 2 * lbo_b) >> 4), idesc,
                     ks > 0);
        tc::mma_commit(tc::smem_u32(&S.bar_pv));
      }
      pv_pending = true;
      pv_ph = ph;
      EA_PT(7)
      // this channel's exponent change, the rows' merges and bounds (registers only) while the P.V
      // MMAs run
      const int ve_now = S.ve[par][c];
      int sh_base[RPT];
      uint64_t ztile[RPT];
#pragma unroll
      for (int ii = 0; ii < RPT; ++ii) {
        const int g = h + NWG * ii;
        sh_base[ii] = INT32_MIN;
        ztile[ii] = 0;
        if (g >= nrows) continue;
        // N in a coarser unit when VE_c grew (this channel) or the row's bound R grows: one floor
        // shift by both (nested floors of divisions compose), its bound ceil-shifted plus one
        int dn = (ve_now != vec && vec != INT32_MIN) ? ve_now - vec : 0;
        const int32_t Rt = max(max(S.rt[0][g], S.rt[1][g]), max(S.rt[2][g], S.rt[3][g]));
        const int32_t Rn = Rt == INT32_MIN ? R[ii] : R[ii] == R_EMPTY ? Rt : max(R[ii], Rt);
        const int dr = (R[ii] != R_EMPTY && Rn > R[ii]) ? Rn - R[ii] : 0;
        dn += dr;
        if (dn > 0) {
          const u128 e = Nerr[ii] + nfl[ii];
          nfl[ii] = 0;
          N[ii] = dn >= 127 ? (N[ii] < 0 ? (i128)-1 : (i128)0) : (N[ii] >> dn);
          Nerr[ii] = (dn >= 128 ? (u128)(e != 0) : (e >> dn) + ((e & ((((u128)1) << dn) - 1)) != 0)) + 1;
        }
        if (Rt == INT32_MIN) continue;
        // Z, its error and the lowest logit are the row's: the channel-0 thread keeps them (it
        // writes them with the partials)
        if (c == 0)
          Tlo[ii] = min(Tlo[ii], min(min(S.rtlo[0][g], S.rtlo[1][g]), min(S.rtlo[2][g], S.rtlo[3][g])));
        if (dr > 0 && c == 0) {
          int lost;
          Z[ii] = floor_shift(Z[ii], -dr, lost);
          Zerr[ii] = scale_ceil(Zerr[ii], -dr) + (uint64_t)lost;
        }
        R[ii] = Rn;
        const uint64_t zt = S.zs[0][g] + S.zs[1][g] + S.zs[2][g] + S.zs[3][g];
        ztile[ii] = zt;
        const uint64_t nlw = (uint64_t)S.zl[0][g] + S.zl[1][g] + S.zl[2][g] + S.zl[3][g];
        if (c == 0) {
          const int zsh = (Rt - FW) - (Rn - FZ);
          int lost = 0;
          Z[ii] += floor_shift((int64_t)zt, zsh, lost);
          Zerr[ii] += (nlw ? scale_ceil(nlw, zsh) : 0) + (uint64_t)lost;
        }
        const int sb = (Rt - FW - FV) - (Rn - FN);
        sh_base[ii] = sb;
        if (nlw) Nerr[ii] += scale_ceil128(nlw, sb + FV);  // truncated weights: < 1 W unit times |v| < 2^VE_c
        // values that lost bits in the V window: their lost parts times the weights, added exactly up
        // to a floor (units 2^(sb - 24)); beyond the list's capacity, the bound of < W + 1 W units
        // times one V unit per such value
        const uint32_t nl = S.vl_n[par][c];
        if (nl == 0) {
        } else if (nl <= VLCAP) {
          i128 corr = 0;
          u128 cerr = 0;
#pragma unroll 1
          for (uint32_t k = 0; k < nl; ++k) {
            const uint32_t ck = S.vl_k[par][c][k];
            const int key = (int)(ck & 0xFFu);
            uint64_t W = 0;
            if (TOEP) {
              W = wval[g * BK + key];
            } else {
#pragma unroll
              for (int wd = 0; wd < NW; ++wd) W |= (uint64_t)sW[tc::kmajor_off(6 * g + wd, key, NSW)] << (8 * wd);
            }
            corr += shift_floor128((i128)(int64_t)W * S.vl_dx[par][c][k], sb - 24);  // 0 <= W dx < 2^72
            cerr += (sb - 24 < 0) ? 1u : 0u;
            if ((ck >> 8) & 1u) cerr += scale_ceil128((u128)W + 1, sb - 24);
          }
          N[ii] += corr;
          Nerr[ii] += cerr;
        } else {
          // more such values than the list holds (or a channel without digits): each lost < 1 V
          // unit (a bounded channel's values are < 2^VE_c: 2^FV units) times < W + 1 W units,
          // bounded over every key of the tile: sum (W + 1) = Z_tile + 128
          Nerr[ii] += scale_ceil128((u128)zt + BK, sb + (nl >= VL_BOUNDED ? FV : 0));
        }
        nfl[ii] += (sb < 0);  // the floor of the tile's one shift into N
      }
      vec = ve_now;
      EA_PT(4)
      // each thread waits; after a wait that gave up the drain reads stale TMEM and the vote at
      // the end of the tile drops it
      const bool ok_pv = tc::mbar_wait(&S.bar_pv, ph, P.wait_debug);
      tc::fence_after_sync();
      EA_PT(5)
      // ---------------- drain: N[g][c] += sum_k 2^(8k) G_k - 2^30 Z_tile, G_k = sum_{u + w = k} D_u[w] ----------------
#pragma unroll
      for (int ii = 0; ii < RPT; ++ii) {
        const int g = h + NWG * ii;
        if (g >= nrows) break;  // uniform across the warp
        uint32_t d0[8], d1[8], d2[8], d3[8];
        int64_t s0, s1, s2, s3, s4, s5, s6, s7, s8;
        if (TOEP) {
          // the digit groups G_0 .. G_8, summed over the four accumulators (each < 4 x 128 x 255
          // x 255 < 2^26 in all)
          // (32-bit sums; two accumulators a wait)
          uint32_t u[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
          for (int a = 0; a < 4; a += 2) {
            tc::tmem_ld8(tlane + COLO + 32 * a + 16 * g, d0);
            tc::tmem_ld2(tlane + COLO + 32 * a + 16 * g + 8, d1);
            tc::tmem_ld8(tlane + COLO + 32 * (a + 1) + 16 * g, d2);
            tc::tmem_ld2(tlane + COLO + 32 * (a + 1) + 16 * g + 8, d3);
            tc::tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 8; ++k) u[k] += d0[k] + d2[k];
            u[8] += d1[0] + d3[0];
          }
          if (sh_base[ii] == INT32_MIN) continue;
          s0 = u[0], s1 = u[1], s2 = u[2], s3 = u[3], s4 = u[4], s5 = u[5], s6 = u[6], s7 = u[7], s8 = u[8];
        } else {
          tc::tmem_ld8(tlane + COLO + 6 * g, d0);
          tc::tmem_ld8(tlane + COLO + NSW + 6 * g, d1);
          tc::tmem_ld8(tlane + COLO + 2 * NSW + 6 * g, d2);
          tc::tmem_ld8(tlane + COLO + 3 * NSW + 6 * g, d3);
          tc::tmem_wait_ld();
          if (sh_base[ii] == INT32_MIN) continue;
          // unsigned digits: 0 <= D_u[w] < 128 keys x 255 x 255 < 2^23, each group (<= 4 terms) < 2^25
          s0 = (int64_t)d0[0];
          s1 = (int64_t)d0[1] + d1[0];
          s2 = (int64_t)d0[2] + d1[1] + d2[0];
          s3 = (int64_t)d0[3] + d1[2] + d2[1] + d3[0];
          s4 = (int64_t)d0[4] + d1[3] + d2[2] + d3[1];
          s5 = (int64_t)d0[5] + d1[4] + d2[3] + d3[2];
          s6 = (int64_t)d1[5] + d2[4] + d3[3];
          s7 = (int64_t)d2[5] + d3[4];
          s8 = (int64_t)d3[5];
        }
        const int64_t lo = s0 + (s1 << 8) + (s2 << 16) + (s3 << 24);  // < 2^50
        const int64_t hi = s4 + (s5 << 8) + (s6 << 16) + (s7 << 24);
        // sum_keys W (x + 2^30) - 2^30 sum_keys W = sum_keys W x, exactly
        const i128 T = (i128)lo + ((i128)hi << 32) + ((i128)s8 << 64) - ((i128)ztile[ii] << 30);
        N[ii] += shift_floor128(T, sh_base[ii]);
      }
      tc::fence_before_sync();
      if (!group_sync_and(BAR_C, NC * 32, ok_pv)) {
        ok_wait = false;
        break;
      }
      pv_pending = false;
      EA_PT(6)
    }
    EA_PT_FLUSH_RANGE(0, 0, 8)
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
  __syncthreads();  // every role is done: row status (also set by the producers) is final
  // ---------------- split partials of this CTA's rows (after every role is done) ----------------
  if (warp < NC) {
#pragma unroll
    for (int ii = 0; ii < RPT; ++ii) {
      const int g = h + NWG * ii;
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
      Nerr[ii] += nfl[ii];
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda)
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)f;
  }
  return fn;
}

// The K fetch mode of a launch and its tensor map: 2D (128 dims x krows rows of bf16), boxes of 64
// dims x `box` rows, 128-byte swizzle. RANGE tiles are 128 consecutive rows; PAGED tiles start on
// page boundaries, so pages of 8..128 keys that divide 128, or multiples of 128, map onto whole
// boxes. Anything else (or a tensor too tall for 32-bit coordinates) takes dense bulk copies.
static int k_fetch_mode(const Prob& P, CUtensorMap* tm, int* kbox) {
  *kbox = 0;
  std::memset(tm, 0, sizeof(*tm));
  int mode = tcd::KM_DENSE, box = 0;
  if (P.kind == MASK_RANGE) {
    mode = tcd::KM_RANGE;
    box = tcd::BK;
  } else if (P.kind == MASK_PAGED && P.page_size > 0) {
    if (P.page_size % tcd::BK == 0) box = tcd::BK;
    else if (tcd::BK % P.page_size == 0 && P.page_size >= 8) box = P.page_size;
    if (box) mode = tcd::KM_PAGED;
  }
  if (mode == tcd::KM_DENSE || P.krows <= 0 || P.krows + tcd::BK >= ((int64_t)1 << 31) || ((uintptr_t)P.k & 15)) return tcd::KM_DENSE;
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return tcd::KM_DENSE;
  const cuuint64_t gdim[2] = {(cuuint64_t)tcd::D, (cuuint64_t)P.krows};
  const cuuint64_t gstride[1] = {(cuuint64_t)tcd::D * 2};
  const cuuint32_t bdim[2] = {64u, (cuuint32_t)box};
  const cuuint32_t estr[2] = {1u, 1u};
  if (enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void*)P.k, gdim, gstride, bdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return tcd::KM_DENSE;
  *kbox = box;
  return mode;
}

// Grid (segments, splits); writes split partials (P.pR ..) for every listed row. max_rows: the
// most rows any segment holds (1..8; 8 when unknown).
cudaError_t launch_tc_decode(const Prob& P, const int32_t* seg_rows, int64_t nseg, int max_rows, cudaStream_t st) {
  // 8 consumer warps with 1, 2 or 4 row slots (segments of <= 2, 4, 8 rows); segments of <= 2
  // rows take 8 K producer warps (640 threads) when the build gives the block the registers its
  // per-role split draws on
  // (RANGE tiles, whose K producers have slack, take two score accumulators; paged ones four:
  // measured on configs 5 and 3)
  auto k0 = tcd::tc_decode_kernel<1, 8, 8>;
  auto k0r = tcd::tc_decode_kernel<1, 8, 8, 2>;
  auto k0s = tcd::tc_decode_kernel<1, 8, 4>;
  auto k1 = tcd::tc_decode_kernel<2, 8, 4>;
  auto k2 = tcd::tc_decode_kernel<4, 8, 4>;
  CUtensorMap tm;
  int kbox = 0;
  const int kmode = k_fetch_mode(P, &tm, &kbox);
  // the shared-memory opt-in is a property of the function on a device: set it once per device
  // (not per launch, so a launch inside a stream capture issues nothing but the kernel)
  static bool attr_set[64][5] = {};
  static int wide_ok = -1;  // the 640-thread kernels' launch registers cover their split (checked once)
  if (wide_ok < 0) {
    cudaFuncAttributes fa, fr;
    wide_ok = cudaFuncGetAttributes(&fa, k0) == cudaSuccess && cudaFuncGetAttributes(&fr, k0r) == cudaSuccess &&
              fa.maxThreadsPerBlock >= tcd::threads_of<8, 8>() && fr.maxThreadsPerBlock >= tcd::threads_of<8, 8>() &&
              fa.numRegs * tcd::threads_of<8, 8>() >= tcd::REG_SPLIT &&
              fr.numRegs * tcd::threads_of<8, 8>() >= tcd::REG_SPLIT;
  }
  const int v = max_rows <= 2 ? (wide_ok ? (kmode == tcd::KM_RANGE ? 4 : 0) : 3) : max_rows <= 4 ? 1 : 2;
  auto kern = v == 0 ? k0 : v == 4 ? k0r : v == 1 ? k1 : v == 2 ? k2 : k0s;
  const bool wide = v == 0 || v == 4;  // the 640-thread kernels: Toeplitz layout
  const int threads = wide ? tcd::threads_of<8, 8>() : tcd::threads_of<8, 4>();
  const int smem = wide ? (int)tcd::T_SMEM_BYTES : (int)tcd::SMEM_BYTES;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev][v]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev][v] = true;
  }
  dim3 grid((unsigned)nseg, (unsigned)P.splits);
  kern<<<grid, threads, smem, st>>>(P, seg_rows, tm, kmode, kbox);
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
