/* Synthetic bf16 workload generator of libexactattn_cuda.so (benchmarks and tests only).
 * Bit-identical to exactattention_b200/workloads.py's numpy generator, so the CPU oracle and the
 * GPU see the same inputs without copying multi-GB tensors. Not part of the attention path; it
 * has no counterpart in the reference, whose benchmarks draw torch.randn on the device. */
#ifndef EXACTATTN_SYNTH_H
#define EXACTATTN_SYNTH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ea_synth {
  uint64_t seed;
  uint64_t tensor_id;
  int64_t G, H, T, D;          /* shape written (groups, heads, tokens, channels) */
  int64_t t0;                  /* first token of the written range within the logical tensor */
  int64_t T_full;              /* tokens of the logical tensor (0: T); element values depend on the
                                  logical index ((g H + h) T_full + t0 + t) D + c only */
  const int32_t* scale_m;      /* (H, D) fp32 scale significands, or NULL for 1.0 */
  const int32_t* scale_e;      /* (H, D) fp32 scale exponents */
  int heavy_permille;          /* rows (g, h, t) scaled by 32 with this probability (per mille) */
  const int32_t* lens;         /* (G,) valid tokens per group, or NULL (all T) */
  const int32_t* page_table;   /* (G, max_pages) or NULL: scatter into (pages, H, page_size, D) */
  int max_pages;
  int page_size;
} ea_synth_t;

/* Fills dst (device memory) on `stream` (a cudaStream_t). Returns 0, -1 bad spec, -4 CUDA error. */
int ea_synth_fill(uint16_t* dst, const ea_synth_t* spec, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EXACTATTN_SYNTH_H */
