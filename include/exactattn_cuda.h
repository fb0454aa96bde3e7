/* C ABI of the B200 (sm_100a) certified ExactAttention library, libexactattn_cuda.so.
 *
 * Every entry point returns bits identical to the spec's (docs/SPEC.md of the reference) or a
 * per-row domain-error flag. Rows that the fast tier cannot certify are recomputed on the GPU
 * (a wide-integer tier); nothing falls back to the CPU.
 *
 * Return codes: 0 OK; -1 bad dimensions; -2 acc_bits not 64/128; -3 non-finite alpha (these
 * three as the reference's csrc/exact_attention_cpu.cpp:589-592); -4 CUDA error; -5 a bounded
 * device wait gave up (a stalled GPU; returned by the synchronous host-pointer entry points after
 * the affected rows were recomputed by the later tiers: out and flags are complete and exact);
 * -6 the allocation-free entry point's scratch is too small for the call; -7 NCCL not found;
 * -8 an NCCL call failed; -9 unsupported layout (mask kind or paged shape).
 * Per-row flags: 0 certified, 2 NaN/inf input or an fp32 logit overflow (the reference raises
 * ExactAttentionDomainError), 1 never expected (no device tier certified the row).
 *
 * Tiers (all on the GPU): tier 1 (tensor-core kernels, or the CUDA-core split kernel) certifies
 * almost every row; the rows it cannot certify are rerun by tier 2 (int64 fixed point on the CUDA
 * cores, each row's keys split into chunks over the whole GPU from a device work list); what
 * tier 2 cannot certify is computed by tier 3 (1536-bit integer windows, also split by key
 * chunks). Value rows wider than 256 channels go straight to tier 3.
 */
#ifndef EXACTATTN_CUDA_H
#define EXACTATTN_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Host-pointer entry point: the drop-in for the reference's
 *   int ea_attention_cpu(const uint16_t* q, int64_t rows, int d, const uint16_t* k,
 *       const uint16_t* v, int64_t nkeys, int dv, float alpha, const int64_t* row_ptr,
 *       const int64_t* key_idx, int fp32_out, int acc_bits, int tile, int splits,
 *       uint64_t order_seed, int nthreads, void* out, uint8_t* flags, int64_t* stats)
 * (reference csrc/exact_attention_cpu.cpp:585-588, bound by src/exactattn/cpu.py:33-41).
 * Same argument order and meaning. q (rows, d), k (nkeys, d), v (nkeys, dv) are bf16 bit
 * patterns; row r attends key_idx[row_ptr[r] .. row_ptr[r+1]) (row_ptr == NULL: every key).
 * acc_bits, tile, order_seed and nthreads are accepted for compatibility: the output does not
 * depend on them. splits partitions each row's keys into KV splits merged exactly.
 * out: rows x dv uint16 (bf16) or float (fp32_out). flags: rows bytes.
 * stats[0..2] += (scores recomputed exactly, weights recomputed with the 128-bit exp2,
 * rows the fast tier left uncertified). Synchronous and thread-safe: the host-pointer entry points share
 * one staging workspace per device, and concurrent calls on one device run one after another. */
int ea_attention_cuda(const uint16_t* q, int64_t rows, int d, const uint16_t* k, const uint16_t* v,
                      int64_t nkeys, int dv, float alpha, const int64_t* row_ptr, const int64_t* key_idx,
                      int fp32_out, int acc_bits, int tile, int splits, uint64_t order_seed, int nthreads,
                      void* out, uint8_t* flags, int64_t* stats);

/* Host-pointer entry point for contiguous key ranges (causal prefill, prefixes, decode):
 * row r attends k rows kv_base[r] .. kv_base[r] + kv_len[r]. The compact form of the CSR mask
 * above (no reference counterpart: the reference's C ABI takes CSR only); same outputs.
 * max_row_keys >= every kv_len[r]. Synchronous; stats as ea_attention_cuda. */
int ea_attention_cuda_ranges(const uint16_t* q, int64_t rows, int d, const uint16_t* k, const uint16_t* v,
                             int64_t nkeys, int dv, float alpha, const int64_t* kv_base, const int64_t* kv_len,
                             int64_t max_row_keys, int fp32_out, int splits, void* out, uint8_t* flags,
                             int64_t* stats);

/* Host-pointer paged decode: q (batch * q_heads, d) with row r = sequence r / q_heads, head
 * r % q_heads; k_cache, v_cache (num_pages, kv_heads, page_size, d / dv); page_table (batch,
 * max_pages) int32; seq_lens (batch,) int32. Staged to the device, synchronous; stats as
 * ea_attention_cuda. The host form of the paged layout of ea_launch_cuda (the reference's C ABI
 * has no paged entry; its paged callers build CSR key lists, which give the same outputs). */
int ea_attention_cuda_paged(const uint16_t* q, int64_t batch, int q_heads, int d, const uint16_t* k_cache,
                            const uint16_t* v_cache, int64_t num_pages, int kv_heads, int page_size, int dv,
                            float alpha, const int32_t* page_table, int max_pages, const int32_t* seq_lens,
                            int fp32_out, int splits, void* out, uint8_t* flags, int64_t* stats);

/* KV-cache write path (paged storage, the layout of EA_MASK_PAGED): append n_new tokens of every
 * (sequence b, kv head h) at positions seq_lens[b] .. seq_lens[b] + n_new - 1; the pages those
 * positions fall in must already be in page_table (the caller's page allocator assigns them).
 * new_k, new_v: (batch, kv_heads, n_new, d) bf16 bits, device pointers, 16-byte aligned; d a
 * multiple of 8 up to 128. advance_lens != 0 adds n_new to seq_lens after the copy (same
 * stream). k_meta (optional, (pages, kv_heads, page_size) uint32): per written key, the largest
 * |k| as bf16 magnitude bits (>= 0x7F80: NaN / inf in the row) | the smallest nonzero |k| << 16
 * (0xFFFF: all zero). The reference slices its cache into int8 planes at this point
 * (triton_kernels.py:1183-1268, 1,053 bytes per key); this library keeps bf16 rows and slices in
 * the kernels. Asynchronous on `stream`. */
typedef struct ea_kv_append {
  uint16_t* k_cache;
  uint16_t* v_cache;
  const int32_t* page_table; /* (batch, max_pages) */
  int32_t* seq_lens;         /* (batch,) */
  const uint16_t* new_k;
  const uint16_t* new_v;
  uint32_t* k_meta; /* optional */
  int64_t batch;
  int kv_heads, page_size, max_pages, n_new, d;
  int advance_lens;
} ea_kv_append_t;
int ea_kv_append_cuda(const ea_kv_append_t* args, void* stream);

/* RN-even of (a / b) * 2^E into fp32 (fp32 != 0) or bf16; a, b given as (hi, lo) 64-bit
 * halves. Mirrors the reference's test export ea_round_ratio
 * (csrc/exact_attention_cpu.cpp:630-638); evaluated on the GPU. */
float ea_round_ratio_cuda(uint64_t a_hi, uint64_t a_lo, uint64_t b_hi, uint64_t b_lo, int E, int neg, int fp32,
                          int* overflow);

/* Mask layouts of the device-pointer entry point. */
/* HYBRID: row r attends kv_base[r] + [0, kv_len[r]) followed by key_idx[row_ptr[r] .. row_ptr[r+1])
 * (a shared prefix plus a per-row list: tree verification). */
enum { EA_MASK_CSR = 0, EA_MASK_RANGE = 1, EA_MASK_PAGED = 2, EA_MASK_HYBRID = 3 };

#define EA_STATS_LEN 12
/* stats slots (int64, accumulated): 0 scores recomputed exactly, 1 weights by the 128-bit exp2,
 * 2 rows tier 1 left uncertified (rerun by tier 2), 3 domain-error rows, 4 unresolved rows
 * (flag 1; never expected), 5 (row, key) pairs processed by tier 1, 6 host fallbacks (always 0),
 * 7 pairs processed by the tensor-core kernels, 8 CTAs whose bounded wait gave up (their rows are
 * recomputed by the later tiers; the host-pointer entry points then return -5), 9 rows tier 2
 * left uncertified (computed by tier 3), 10 (row, key) pairs rerun by tier 2, 11 rows the test
 * hook forced out of tier 1. */

typedef struct ea_launch {
  /* inputs, device pointers */
  const uint16_t* q; /* (rows, d) */
  int64_t rows;
  int d;
  const uint16_t* k; /* key rows of d values (CSR/RANGE: (nkeys, d); PAGED: (pages, kv_heads, page_size, d)) */
  const uint16_t* v; /* value rows of dv values, same row indexing as k */
  int64_t nkeys;
  int dv;
  float alpha;
  /* mask */
  int mask_kind;
  const int64_t* row_ptr; /* CSR: rows + 1 */
  const int64_t* key_idx; /* CSR */
  const int64_t* kv_base; /* RANGE: row r attends k rows kv_base[r] .. kv_base[r] + kv_len[r] */
  const int64_t* kv_len;
  const int32_t* page_table; /* PAGED: (batch, max_pages) physical page ids */
  const int32_t* seq_lens;   /* PAGED: (batch,) keys per sequence */
  int page_size, max_pages, q_heads, kv_heads; /* PAGED: row r = seq (r / q_heads), head r % q_heads */
  int64_t max_row_keys; /* >= every row's key count (sets the fixed-point headroom) */
  int fp32_out;
  int splits;
  /* outputs, device pointers */
  void* out;      /* (rows, dv) uint16 or float */
  uint8_t* flags; /* (rows,) */
  int64_t* stats; /* EA_STATS_LEN int64 counters, accumulated; may be NULL */
  /* optional, RANGE and HYBRID masks: every row in one of the blocks of 128 rows that share
   * kv_base (-1 pads a block), (nblocks, 128) int32. With it and d = dv = 128 (bf16 or fp32
   * output), the tensor-core kernel runs (RANGE: when splits == 1; HYBRID: over the range part,
   * with the per-row lists on the CUDA cores); any grouping gives the same bits. */
  const int32_t* block_rows;
  int64_t nblocks;
  /* optional, RANGE masks (decode): segments of up to 8 rows that share kv_base (-1 pads),
   * (nsegs, 8) int32, every row in one segment. With it, d = dv = 128, the tensor-core decode
   * kernel runs: keys on the MMA's M side, the segment's rows in N, `splits` CTAs per segment.
   * PAGED masks with d = dv = 128 and q_heads / kv_heads <= 8 take that kernel without it. */
  const int32_t* seg_rows;
  int64_t nsegs;
  /* optional: the most rows any segment of seg_rows holds (1..8; 0 = up to 8). Segments of a GQA
   * group of 2 (or 4) let the decode kernel keep fewer running sums per thread. */
  int seg_width;
} ea_launch_t;

/* Device-pointer entry point: asynchronous on `stream` (a cudaStream_t, NULL = default).
 * Uses a library-owned workspace on the current device (grown outside any stream capture by
 * ea_reserve_workspace or on first use). The device-pointer entry points of one device share it
 * (split partials, tier-3 work list): launches on different streams of one device must be ordered
 * (one stream, or events between streams), as with one cuBLAS handle. The host-pointer entry
 * points use a workspace of their own. The torch-tensor API builds on this. */
int ea_launch_cuda(const ea_launch_t* args, void* stream);

/* Per-row partial state of one key range (the split partial of the reference's certified
 * split-KV kernel, src/exactattn/triton_kernels.py:731 _split_program and _ea_combine_kernel
 * :1081, and certified.py:213 `merge`), exported to device buffers so that partials computed on
 * different GPUs can be merged. All device pointers; rows x dv for NR, N, Nerr.
 *   R       row exponent: Z = Z_int * 2^(R - FZ); INT32_MIN for a row with no keys
 *   Z, Zerr lower bound of the weight sum and its nonnegative error, in units 2^(R - FZ)
 *   status  0 certified so far, 1 needs the exact tier (tier 3), 2 domain error
 *   NR      per-channel exponent of the numerator (INT32_MIN: no contribution)
 *   N, Nerr lower bound of the numerator and its error, units 2^(NR - FZ)
 * FZ = 61 - ceil(log2(max_row_keys)) for the launch's max_row_keys (must be the same on every
 * rank). Merging: R_g = max over ranks of R, NR_g = max of NR, status = max of status; every
 * rank rescales to (R_g, NR_g) with ea_partials_rescale_cuda (floor shifts, error grown by one
 * unit per shifted value); then Z, Zerr, N, Nerr are summed over ranks; the sum is finalised
 * by ea_partials_finalize_cuda. Every step is order independent, so any all-reduce tree gives
 * the same bits. No reference counterpart as a separate entry point: the reference merges
 * split partials inside one launch (triton_kernels.py:1081 _ea_combine_kernel). */
typedef struct ea_partials {
  int32_t* R;
  int64_t* Z;
  int64_t* Zerr;
  int32_t* status;
  int32_t* NR;
  int64_t* N;
  int64_t* Nerr;
} ea_partials_t;

/* Tier-1 pass of `args` (any mask, any splits; the tensor-core kernel where it applies) that
 * writes the row partials instead of outputs. args->out/flags are not written. */
int ea_partials_cuda(const ea_launch_t* args, const ea_partials_t* parts, void* stream);
/* In-place rescale of `parts` to the global exponents R_global (rows) and NR_global (rows x dv). */
int ea_partials_rescale_cuda(const ea_partials_t* parts, const int32_t* R_global, const int32_t* NR_global,
                             int64_t rows, int dv, void* stream);
/* Certified rounding of merged partials into out/flags (flag 1: not certifiable from the merged
 * interval, the row needs the wide tier below, counted in stats[2]; flag 2: domain error). */
int ea_partials_finalize_cuda(const ea_partials_t* parts, int64_t rows, int dv, int64_t max_row_keys,
                              int fp32_out, void* out, uint8_t* flags, int64_t* stats, void* stream);

/* The one-collective form of the KV-shard merge. Each rank keeps its partials in one flat buffer
 * of EA_PARTIALS_FLAT_BYTES(rows, dv) bytes (int64 Z[rows], Zerr[rows], N[rows dv], Nerr[rows dv],
 * then int32 R[rows], status[rows], NR[rows dv], padded to a multiple of 8 bytes; an ea_partials_t
 * pointing into it is filled by ea_partials_cuda as usual). After an all-gather of those buffers
 * (rank order does not matter), `gathered` holds world buffers back to back; this merges them (MAX
 * of the exponents, every partial re-expressed at them, SUM: order-free) and rounds every row,
 * writing out and flags on every rank alike. Rows the merged interval cannot certify get flag 1 and
 * are listed in increasing row order in wide_rows (capacity rows; every slot past the count holds
 * -1; the count in the device int *wide_count), the same list on every rank, for the sharded wide
 * tier (ea_wide_partials_cuda and the following entries, which pair the ranks' partials slot by
 * slot). Replaces
 * ea_partials_rescale_cuda + a SUM all-reduce + ea_partials_finalize_cuda: one collective instead of
 * two, one kernel. No reference counterpart (the reference runs on one device). */
#define EA_PARTIALS_FLAT_BYTES(rows, dv) \
  ((((size_t)(rows) * (16 + 16 * (size_t)(dv)) + (size_t)(rows) * (8 + 4 * (size_t)(dv))) + 7) & ~(size_t)7)
int ea_partials_merge_gathered_cuda(const void* gathered, int world, int64_t rows, int dv, int64_t max_row_keys,
                                    int fp32_out, void* out, uint8_t* flags, int32_t* wide_rows, int32_t* wide_count,
                                    int64_t* stats, void* stream);

/* The whole KV-shard merge of `parts` over the caller's NCCL communicator (an ncclComm_t passed
 * as void*), on `stream`: all-reduce MAX of R, status and NR, ea_partials_rescale_cuda, all-reduce
 * SUM of Z, Zerr, N and Nerr; then ea_partials_finalize_cuda gives every rank the same rows. Every
 * rank calls it with the same rows and dv (also rows = 0). NCCL (libnccl.so.2) is loaded at run
 * time, preferring a copy the process already loaded, so the communicator must come from that
 * library. Returns 0, -1 bad arguments, -4 CUDA error, -7 NCCL not found, -8 an NCCL call failed.
 * Calls on one device share a scratch array (rows x (dv + 1) int32), so they are ordered like
 * ea_launch_cuda's. The Python form is exactattention_b200/dist.py (torch.distributed). No reference counterpart
 * (the reference runs on one device). */
int ea_merge_partials_nccl(const ea_partials_t* parts, int64_t rows, int dv, void* nccl_comm, void* stream);

/* Wide (tier-3) partials for the rows ea_partials_finalize_cuda flagged 1, so that KV-sharded
 * runs finish every row on the devices. Per listed row i (device pointers):
 *   maxv[4 i + 0..3]  R (reference exponent, INT64_MIN: no keys), Emax, -Emin (weight exponent
 *                     range), status; merged by MAX over ranks
 *   sumv[((dv + 1) i + j) (EA_WIDE_DIGITS + 1) + ..]  j = 0: Z, j = 1 + c: channel c's N, as
 *                     EA_WIDE_DIGITS signed 32-bit digits in int64 followed by the error bound;
 *                     merged by SUM over ranks after ea_wide_partials_rescale_cuda.
 * Merge: copy maxv, all-reduce MAX the copy (merged_max), rescale with it, all-reduce SUM sumv,
 * finalise with merged_max. `rows` (n int32 row indices) must be the same on every rank. These
 * carry the reference's exact big-integer sums (reference.py:146 attention_row) across devices; no
 * reference counterpart as an entry point. */
#define EA_WIDE_DIGITS 48
typedef struct ea_wide_partials {
  int64_t* maxv;
  int64_t* sumv;
} ea_wide_partials_t;
int ea_wide_partials_cuda(const ea_launch_t* args, const int32_t* rows, int n, const ea_wide_partials_t* parts,
                          void* stream);
int ea_wide_partials_rescale_cuda(const ea_wide_partials_t* parts, const int64_t* merged_max, int n, int dv,
                                  void* stream);
/* Writes out/flags of the listed rows: flag 0 certified, 2 domain error, 1 unresolved (a
 * 2^-97-probability event; counted in stats[4]). A row index below 0 in `rows` marks an unused slot
 * of a fixed-capacity list (an empty partial, nothing written): a caller can then run these calls
 * with a fixed n every step, without reading the wide-row count on the host. */
int ea_wide_partials_finalize_cuda(const ea_wide_partials_t* parts, const int64_t* merged_max, const int32_t* rows,
                                   int n, int dv, int fp32_out, void* out, uint8_t* flags, int64_t* stats,
                                   void* stream);

/* Diagnostic timing of the hot kernel: mode 1 switches it on (and clears it; no more than 512
 * launches are recorded), mode 2 waits for the recorded launches and returns the summed device
 * time (ms) of their tier-1 kernel (tensor-core prefill or decode, or the CUDA-core split kernel)
 * and the count, then clears; mode 0 switches it off. CUDA events are recorded on the launch
 * stream around that kernel. No reference counterpart (a measurement hook of this library). */
int ea_kernel_timing(int mode, double* total_ms, int64_t* launches);

/* Self-test of the binary64 fast paths of the per-pair roundings against their exact integer
 * evaluations, on the current device (no reference counterpart: the reference has one exact
 * evaluation). mode 0: weights RN24(2^t) for n logits t, fp32 bit patterns from `seed` with step
 * `stride`, both signs, |t| < 2^22; mode 1: logits RN32(alpha s) for n splitmix64 cases from
 * `seed`; mode 2: output ratios RN(a / b 2^sh) to bf16 and fp32 for n splitmix64 cases; mode 3:
 * the same ratios through one reciprocal of b (the form the prefill kernel uses per row).
 * out[0..3] = cases, cases the fast path certified, mismatches (must be 0), the input of a
 * mismatch. Returns 0, or -1 / -4 for bad arguments / a CUDA error. */
int ea_selftest_fast64(int mode, uint64_t seed, uint32_t stride, int64_t n, int64_t* out);

/* Allocation-free form of ea_launch_cuda, for callers that cannot allocate device memory when
 * they run attention: a serving process whose memory pool owns the whole GPU and forbids
 * allocations behind its back, or a latency-bound loop that cannot stall on a first cudaMalloc.
 * No counterpart in the reference. Its scratch (split partials, tier-3 work list, counters) is one
 * static device array of EA_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps until
 * exit. A call needs, with A(x) = x rounded up to a multiple of 256 and n = rows x splits,
 *   A(8 EA_STATS_LEN) + A(4) + A(4 rows)
 *   + (splits > 1 ? 2 A(8 n) + 2 A(8 n dv) + 2 A(4 n) + A(4 n dv) : 0)
 * bytes; a call needing more returns -6. Every failure's message is in ea_noalloc_last_error().
 * The first call on a device looks up the array's address (cudaGetSymbolAddress with that device
 * current): make that first call before any stream capture. Calls share the array, which keeps the
 * previous call's contents (each call clears what must start at zero), so calls on one device
 * whose kernels may overlap race and must be serialised. CUDA-core kernels only (d <= 1024,
 * dv <= 256, splits <= 65535); the test hooks do not apply. */
#define EA_NOALLOC_SCRATCH_BYTES (32u << 20)
int ea_attention_cuda_noalloc(const ea_launch_t* args, void* stream);
const char* ea_noalloc_last_error(void);

/* The EA_STATS_LEN counters of the calling thread's last successful host-pointer call
 * (ea_attention_cuda, _ranges, _paged): the reference's C entry reports three counters through its
 * `stats` argument; this gives the rest (pairs on the tensor cores, tier-2 work, ...). No reference
 * counterpart. Returns 0, or -1 for a NULL out. */
int ea_last_host_stats(int64_t* out);

/* Test hooks, for tests of this library (all zero in production). force_stride > 0: every row r
 * with r % force_stride == 0 that tier 1 certified is treated as uncertified, so it runs through
 * tier 2, and with force_tier == 2 through tier 3 as well (stats[11] counts the rows); the output
 * bits must not change. wait_debug != 0: every bounded wait of the tensor-core kernels reports
 * expiry once its phase has completed (or after 20 ms), so their abort path runs with nothing left
 * in flight: stats[8] counts the CTAs, their rows are recomputed by the later tiers, and the
 * host-pointer entry points return -5. Applies to every device, to launches made after the call;
 * NULL resets. Returns 0 or -1. No reference counterpart as an entry point: the reference drives
 * its fallback tiers in tests by narrowing its windows (Config(acc_bits=34),
 * tests/test_certified.py:129-139). */
typedef struct ea_test_hooks {
  int force_stride;
  int force_tier;
  int wait_debug;
} ea_test_hooks_t;
int ea_set_test_hooks(const ea_test_hooks_t* hooks);

/* Sizes the workspace for up to `rows` rows, `splits` splits and dv channels on the current
 * device; call before capturing a launch in a CUDA graph. */
int ea_reserve_workspace(int64_t rows, int splits, int dv);

/* Frees the workspace of every device. */
void ea_cuda_release(void);

/* Last CUDA error string of this library (thread-local). */
const char* ea_cuda_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* EXACTATTN_CUDA_H */
