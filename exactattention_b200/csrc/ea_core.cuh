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
  STAT_TIER3_ROWS = 2,    // rows sent to the wide-integer tier
  STAT_DOMAIN_ROWS = 3,   // rows flagged 2 (NaN/inf input, logit overflow, exponent spread)
  STAT_UNRESOLVED = 4,    // rows no device tier certified (never expected; flagged 1)
  STAT_PAIRS = 5,         // (row, key) pairs processed by tier 1
  STAT_HOST_FALLBACKS = 6,// always 0: there is no host fallback
  STAT_TC_PAIRS = 7,      // pairs whose scores and P.V ran on the tensor cores
  STAT_LEN = 8
};

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
  int* t3_count;
  int* t3_list;
  int t3_fixed;  // > 0: number of listed rows (instead of *t3_count)
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

}  // namespace ea
