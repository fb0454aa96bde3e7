// KV-cache write path: append new keys / values of every (sequence, kv head) into paged storage,
// optionally with a per-key summary of the K row that the certified kernels can use.
//
// The reference slices K and V into int8 digit planes when its cache is written
// (src/exactattn/triton_kernels.py:1183-1268 tc_slices / tc_v_slices, 1,053 bytes per key). This
// library keeps the cache in bf16 (512 bytes per key and kv head for d = 128) and cuts digits
// inside the attention kernels, so the write path only places rows; the summary kept per key is
// 4 bytes: the largest |k| as bf16 magnitude bits (0x7F80 or more: a NaN / inf in the row) and the
// smallest nonzero |k| (0xFFFF: no nonzero element), from which a kernel knows the row's block
// exponent and whether any element falls below its window without reading the row first.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/exactattn_cuda.h"

namespace ea {
namespace {

// Thread per (sequence, kv head, new token, 8 elements): one 16-byte load and store each for K and
// V; the 16 lanes of a row reduce its magnitudes for the summary.
__global__ void kv_append_kernel(ea_kv_append_t a) {
  const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = a.d / 8;
  const int64_t total = (int64_t)a.batch * a.kv_heads * a.n_new * per_row;
  const bool valid = item < total;
  const int64_t r = valid ? item / per_row : 0;  // (b, h, j) row
  const int c8 = (int)(item - r * per_row);
  const int j = (int)(r % a.n_new);
  const int h = (int)((r / a.n_new) % a.kv_heads);
  const int b = (int)(r / ((int64_t)a.n_new * a.kv_heads));
  uint32_t mx = 0, mn = 0xFFFFu;
  int64_t dst_row = 0;
  if (valid) {
    const int64_t pos = (int64_t)a.seq_lens[b] + j;
    const int64_t page = a.page_table[(int64_t)b * a.max_pages + pos / a.page_size];
    dst_row = (page * a.kv_heads + h) * a.page_size + pos % a.page_size;
    const uint4 kx = ((const uint4*)(a.new_k + r * a.d))[c8];
    const uint4 vx = ((const uint4*)(a.new_v + r * a.d))[c8];
    ((uint4*)(a.k_cache + dst_row * a.d))[c8] = kx;
    ((uint4*)(a.v_cache + dst_row * a.d))[c8] = vx;
    const uint32_t w[4] = {kx.x, kx.y, kx.z, kx.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t m = (w[i] >> (16 * hh)) & 0x7FFFu;
        mx = max(mx, m);
        if (m) mn = min(mn, m);
      }
  }
  if (a.k_meta) {
    // lanes of one row are consecutive: per_row (<= 16 for d <= 128) divides 32
    for (int o = 1; o < per_row; o <<= 1) {
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    }
    if (valid && c8 == 0) a.k_meta[dst_row] = mx | (mn << 16);
  }
}

__global__ void seq_lens_add_kernel(int32_t* seq_lens, int64_t batch, int n_new) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) seq_lens[b] += n_new;
}

}  // namespace
}  // namespace ea

extern "C" int ea_kv_append_cuda(const ea_kv_append_t* a, void* stream) {
  if (!a || a->batch < 0 || a->kv_heads <= 0 || a->n_new < 0 || a->page_size <= 0 || a->max_pages <= 0) return -1;
  if (a->d <= 0 || a->d % 8 != 0 || a->d > 128 || (32 % (a->d / 8)) != 0) return -5;  // rows of 16-byte pieces
  if (((uintptr_t)a->k_cache | (uintptr_t)a->v_cache | (uintptr_t)a->new_k | (uintptr_t)a->new_v) & 15) return -5;
  if (a->batch == 0 || a->n_new == 0) return 0;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t items = (int64_t)a->batch * a->kv_heads * a->n_new * (a->d / 8);
  ea::kv_append_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(*a);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && a->advance_lens)
    ea::seq_lens_add_kernel<<<(unsigned)((a->batch + 255) / 256), 256, 0, st>>>(a->seq_lens, a->batch, a->n_new);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -4;
}
