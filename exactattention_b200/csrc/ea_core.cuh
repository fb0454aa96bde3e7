// Problem description, key addressing and per-row finalisation shared by the CUDA kernels of
// certified ExactAttention.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ea_numerics.h"

namespace ea {

// How row r's j-th key maps to a row of K (d values) and of V (dv values).
// HYBRID: a contiguous range (RANGE) followed by a CSR list (tree verification: prefix + ancestors).
enum MaskKind { MASK_CSR = 0, MASK_RANGE = 1, MASK_PAGED = 2, MASK_HYBRID = 3 };

// Per (row, split) status; the final per-row flag is 0 (certified at some device tier) or 2.
enum Status { ST_OK = 0, ST_TIER3 = 1, ST_DOMAIN = 2 };

constexpr int32_t R_EMPTY = INT32_MIN;
// The reference refuses rows whose weight exponents spread over more than 2^20
// (reference.py:30, 116-118). Tier 1 sends a row to tier 3 (which decides the spread exactly)
// when one unit of work sees its logits span more than SPREAD_CHECK (R - lowest floor(t)), and
// the merge of units does when a unit's R lies more than SPREAD_CHECK below the row's: together
// these cover every spread above 2^20 - 16. A KV shard marks a far-below partial by adding
// SPREAD_MARK to its Zerr (a legitimate Zerr stays below 2^40), which survives the sum.
constexpr int32_t SPREAD_CHECK = (1 << 19) - 8;
constexpr uint64_t SPREAD_MARK = 1ull << 56;

// Device statistics counters (accumulated, never reset by a launch).
enum Stat {
  STAT_SCORE_EXACT = 0,   // (row, key) scores the window could not certify: recomputed exactly
  STAT_WEIGHT_WIDE = 1,   // weights the 64-bit exp2 could not certify: 128-bit exp2
  STAT_TIER1_UNCERT = 2,  // rows tier 1 left uncertified (rerun by tier 2)
  STAT_DOMAIN_ROWS = 3,   // rows flagged 2 (NaN/inf input, logit overflow, exponent spread)
  STAT_UNRESOLVED = 4,    // rows no device tier certified (never expected; flagged 1)
  STAT_PAIRS = 5,         // (row, key) pairs processed by tier 1
  STAT_HOST_FALLBACKS = 6,// always 0: there is no host fallback
  STAT_TC_PAIRS = 7,      // pairs whose scores and P.V ran on the tensor cores
  STAT_WAIT_EXPIRED = 8,  // CTAs of a tensor-core kernel whose bounded wait gave up
  STAT_TIER2_UNCERT = 9,  // rows tier 2 left uncertified (sent to the wide tier 3)
  STAT_TIER2_PAIRS = 10,  // (row, key) pairs rerun by tier 2
  STAT_FORCED_ROWS = 11,  // rows the test hook declared uncertified
  STAT_LEN = 12
};
// the tier-1 name of slot 2 before tier 2 existed
constexpr int STAT_TIER3_ROWS = STAT_TIER1_UNCERT;

struct Prob {
  // inputs
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  int64_t rows;
  int d, dv;
  int W;           // q/k block fixed-point window (bits)
  int32_t am, ae;  // alpha = am * 2^ae
  int fp32;
  // mask
  int kind;
  const int64_t* row_ptr;
  const int64_t* key_idx;
  const int64_t* kv_base;
  const int64_t* kv_len;
  const int32_t* page_table;
  const int32_t* seq_lens;
  int page_size, max_pages, hq, group, hkv;
  int64_t krows;  // rows of the K (and V) tensor: keys (CSR / RANGE) or pages x kv heads x page size
  // schedule / headroom
  int splits;
  int key_log2;
  int FZ;          // fraction bits of the int64 Z and N windows: 61 - key_log2
  // outputs
  void* out;
  uint8_t* flags;
  // split partials (splits > 1)
  int32_t* pR;
  int64_t* pZ;
  uint64_t* pZe;
  int32_t* pSt;
  int32_t* pNR;
  int64_t* pN;
  uint64_t* pNe;
  // export: write one partial per row instead of finalising (KV-sharded runs merge them across
  // GPUs). Layout of ea_partials_t; N is one-sided: the value lies in [N, N + Nerr] units.
  int export_partials;
  int32_t* xR;
  int64_t* xZ;
  uint64_t* xZe;
  int32_t* xSt;
  int32_t* xNR;
  int64_t* xN;
  uint64_t* xNe;
  // wide (tier-3) partials of the rows in t3_list, when export_partials is set for tier 3:
  // w3max (n x 4, merged by MAX): R, Emax, -Emin, status; w3sum (n x (dv + 1) x (LW + 1),
  // merged by SUM): Z's LW digits and Zerr, then each channel's N digits and Nerr
  int64_t* w3max;
  int64_t* w3sum;
  // bookkeeping
  unsigned long long* stats;
  int* t3_count;  // rows the running tier leaves uncertified are appended to (t3_list, t3_count)
  int* t3_list;
  int t3_fixed;  // > 0: number of listed rows (instead of *t3_count)
  // split-K units of tier 2 / tier 3: listed row i covers units u_off[i] .. u_off[i + 1], unit k
  // of a row its keys [k chunk, (k + 1) chunk); the values live in device memory (set by a plan
  // kernel, so no host synchronisation): u_off (n + 1), u_n = {rows, units, chunk}
  const int* u_off;
  const int64_t* u_n;
  const int* u_rows;  // the listed rows of the plan
  // tier: 1 tier 1 (its uncertified rows go to tier 2, or straight to tier 3 without one), 2 tier 2
  int tier;
  // test hooks (ea_set_test_hooks; 0 in production): rows r with r % force_stride == 0 are
  // treated as uncertified by tier 1, and by tier 2 too when force_tier >= 2; wait_debug != 0
  // makes every bounded wait of the tensor-core kernels report expiry once its phase completed
  // (or after a short limit), which exercises the abort path
  int force_stride, force_tier, wait_debug;
};

__device__ __forceinline__ int64_t row_len(const Prob& P, int64_t r) {
  if (P.kind == MASK_CSR) return P.row_ptr[r + 1] - P.row_ptr[r];
  if (P.kind == MASK_RANGE) return P.kv_len[r];
  if (P.kind == MASK_HYBRID) return P.kv_len[r] + (P.row_ptr[r + 1] - P.row_ptr[r]);
  return (int64_t)P.seq_lens[r / P.hq];
}

// index of the K row (and V row) of row r's j-th key
__device__ __forceinline__ int64_t key_row(const Prob& P, int64_t r, int64_t j) {
  if (P.kind == MASK_CSR) return P.key_idx[P.row_ptr[r] + j];
  if (P.kind == MASK_RANGE) return P.kv_base[r] + j;
  if (P.kind == MASK_HYBRID) {
    int64_t n0 = P.kv_len[r];
    return j < n0 ? P.kv_base[r] + j : P.key_idx[P.row_ptr[r] + (j - n0)];
  }
  int64_t b = r / P.hq;
  int h = (int)(r - b * P.hq);
  int kvh = h / P.group;
  int64_t page = P.page_table[b * P.max_pages + j / P.page_size];
  return (page * P.hkv + kvh) * P.page_size + (j % P.page_size);
}

__device__ __forceinline__ void stat_add(const Prob& P, int which, unsigned long long n) {
  if (n) atomicAdd(P.stats + which, n);
}

__device__ __forceinline__ void write_out(const Prob& P, int64_t r, int c, const Rnd& x) {
  if (P.fp32)
    ((uint32_t*)P.out)[r * P.dv + c] = rnd_to_f32_bits(x);
  else
    ((uint16_t*)P.out)[r * P.dv + c] = (uint16_t)rnd_to_bf16_bits(x);
}

__device__ __forceinline__ void push_tier3(const Prob& P, int64_t r) {
  int i = atomicAdd(P.t3_count, 1);
  P.t3_list[i] = (int)r;
}

// A row that this tier could not certify goes on to the next one (counted per tier).
__device__ __forceinline__ void push_uncertified(const Prob& P, int64_t r) {
  push_tier3(P, r);
  stat_add(P, P.tier == 2 ? STAT_TIER2_UNCERT : STAT_TIER1_UNCERT, 1);
}

// The test hook: this certified row is to be treated as uncertified by the running tier (the
// caller counts it once in STAT_FORCED_ROWS at tier 1).
__device__ __forceinline__ bool forced_uncertified(const Prob& P, int64_t r) {
  if (P.force_stride <= 0 || r % P.force_stride != 0) return false;
  return P.tier != 2 || P.force_tier >= 2;
}

// The row leaves this tier uncertified: by its own bounds (forced = false) or the test hook.
__device__ __forceinline__ void leave_tier(const Prob& P, int64_t r, bool forced) {
  push_uncertified(P, r);
  if (forced && P.tier != 2) stat_add(P, STAT_FORCED_ROWS, 1);
}

// Device buffers of the fallback tiers (one set per workspace; sized by fallback_bytes).
// Tier 2: at most T2_MAX_ROWS rows per launch (the rest go straight to tier 3), their keys cut
// into at most T2_UNITS units; tier 3: split by key chunks into at most T3_UNITS units when
// T3_SPLIT_ROWS rows or fewer are left, otherwise one block per row.
constexpr int T2_MAX_ROWS = 4096, T2_UNITS = 8192, T3_SPLIT_ROWS = 256, T3_UNITS = 512;
constexpr int64_t T2_MIN_CHUNK = 256, T3_MIN_CHUNK = 1024;
struct FallbackBufs {
  int* list3;      // rows tier 2 leaves uncertified (tier 3's list), capacity: the launch's rows
  int* count3;
  int* u2_off;     // T2_MAX_ROWS + 1
  int64_t* u2_n;   // 4
  int* u3_off;     // T3_SPLIT_ROWS + 1
  int64_t* u3_n;   // 4
  int64_t* g3;     // T3_SPLIT_ROWS x 4: merged maxima of tier 3's split rows
  // tier-2 unit partials (T2_UNITS slots, the split-partial layout)
  int32_t* pR;
  int64_t* pZ;
  uint64_t* pZe;
  int32_t* pSt;
  int32_t* pNR;
  int64_t* pN;
  uint64_t* pNe;
  int32_t* pRlo;  // a merged group's lowest exponent, at its head slot (the spread check)
  // tier-3 unit wide partials (T3_UNITS slots)
  int64_t* w3max;
  int64_t* w3sum;
};

}  // namespace ea
