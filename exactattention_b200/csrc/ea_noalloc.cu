// ea_attention_cuda_noalloc: the device-pointer entry point without any device allocation.
//
// Some callers cannot allocate device memory at the moment they need attention: serving
// processes whose memory pool owns the whole device and forbids allocations behind its back,
// and latency-bound decode loops that cannot afford the stall (and the implicit device
// synchronisation) of a first-call cudaMalloc. This entry point serves them: the split
// partials, the tier-3 work list and the counters live in one file-scope __device__ array of
// fixed size, reserved when the library is loaded (every GPU that loads the library keeps it
// until exit).
//
// Limits and rules:
//   * the scratch holds EA_NOALLOC_SCRATCH_BYTES; a call that needs more (the exact formula is in
//     scratch_bytes below and in include/exactattn_cuda.h) is rejected with -6 and an error
//     string, before anything is launched;
//   * the first call on a device looks up the array's device address (cudaGetSymbolAddress)
//     with that device current; make that first call before any stream capture;
//   * every call uses the same array and it keeps the previous call's contents: the counters
//     that must start at zero are cleared by each call, on the caller's stream;
//   * two calls on the same device whose kernels can run at the same time (different streams,
//     or different host threads without ordering) race on the array: serialise them. Calls on
//     different devices use different copies of the array.
// Only the CUDA-core kernels run here (every mask, any d <= 1024 and dv <= 256); the tensor-core
// kernel is not used.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <string>

#include "../../include/exactattn_cuda.h"
#include "ea_core.cuh"

namespace ea {
cudaError_t launch_simt(const Prob& P, cudaStream_t st);
cudaError_t launch_tier3(const Prob& P, int blocks, cudaStream_t st);
}  // namespace ea

using namespace ea;

namespace {

// The scratch array. In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory: only the address from cudaGetSymbolAddress may be given to a kernel.
static __device__ __align__(256) unsigned char g_noalloc_scratch[EA_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
unsigned char* g_scratch_ptr[MAX_DEVICES] = {};
int g_sms[MAX_DEVICES] = {};
thread_local std::string g_err;

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// bytes of scratch one call needs (same layout as the carve-up below); callers have checked
// rows <= SCRATCH / 4 and rows x splits <= SCRATCH / 4, so no product here overflows
size_t scratch_bytes(int64_t rows, int splits, int dv) {
  size_t b = align256(EA_STATS_LEN * 8) + align256(sizeof(int)) + align256((size_t)rows * 4);
  if (splits > 1) {
    size_t n = (size_t)rows * splits;
    b += 2 * align256(n * 8) + 2 * align256(n * dv * 8) + 2 * align256(n * 4) + align256(n * dv * 4);
  }
  return b;
}

int ceil_log2(int64_t n) {
  int k = 0;
  while (((int64_t)1 << k) < n) ++k;
  return k;
}

}  // namespace

extern "C" const char* ea_noalloc_last_error(void) { return g_err.c_str(); }

extern "C" int ea_attention_cuda_noalloc(const ea_launch_t* a, void* stream) {
  if (!a || a->d <= 0 || a->d > 1024 || a->dv <= 0 || a->dv > 256 || a->splits <= 0 || a->splits > 65535 ||
      a->rows < 0) {
    g_err = "ea_attention_cuda_noalloc: invalid dimensions (d <= 1024, dv <= 256, 1 <= splits <= 65535)";
    return -1;
  }
  uint32_t ab;
  memcpy(&ab, &a->alpha, 4);
  int32_t am, ae;
  if (!decode_fp32(ab, am, ae)) {
    g_err = "ea_attention_cuda_noalloc: alpha is not finite";
    return -3;
  }
  if (a->mask_kind < EA_MASK_CSR || a->mask_kind > EA_MASK_HYBRID ||
      (a->mask_kind == EA_MASK_PAGED && (a->page_size <= 0 || a->q_heads <= 0 || a->kv_heads <= 0 ||
                                         a->q_heads % a->kv_heads != 0))) {
    g_err = "ea_attention_cuda_noalloc: unsupported layout";
    return -9;
  }
  if (a->rows == 0) return 0;
  // every row takes 4 bytes of the work list and every (row, split) at least 4 bytes of
  // partials: bounding both first keeps the size arithmetic below free of overflow
  constexpr int64_t cap4 = (int64_t)EA_NOALLOC_SCRATCH_BYTES / 4;
  const bool too_many = a->rows > cap4 || (a->splits > 1 && a->rows > cap4 / a->splits);
  const size_t need = too_many ? 0 : scratch_bytes(a->rows, a->splits, a->dv);
  if (too_many || need > (size_t)EA_NOALLOC_SCRATCH_BYTES) {
    g_err = "ea_attention_cuda_noalloc: needs " + (too_many ? std::string("more") : std::to_string(need)) +
            " bytes of scratch, the maximum is " + std::to_string((size_t)EA_NOALLOC_SCRATCH_BYTES) +
            " (use fewer rows or splits per call)";
    return -6;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
    g_err = "ea_attention_cuda_noalloc: no current CUDA device";
    return -4;
  }
  unsigned char* base;
  int sms;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
      // once per device, with that device current: the device address of the scratch array
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        g_err = std::string("ea_attention_cuda_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e);
        return -4;
      }
      int n = 148;
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
      g_sms[dev] = n;
      g_scratch_ptr[dev] = (unsigned char*)p;
    }
    base = g_scratch_ptr[dev];
    sms = g_sms[dev];
  }
  cudaStream_t st = (cudaStream_t)stream;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* r = base + off;
    off += align256(bytes);
    return (void*)r;
  };
  Prob P;
  memset(&P, 0, sizeof(P));
  unsigned long long* stats = (unsigned long long*)take(EA_STATS_LEN * 8);
  P.t3_count = (int*)take(sizeof(int));
  P.t3_list = (int*)take((size_t)a->rows * 4);
  if (a->splits > 1) {
    const size_t n = (size_t)a->rows * a->splits;
    P.pZ = (int64_t*)take(n * 8);
    P.pZe = (uint64_t*)take(n * 8);
    P.pN = (int64_t*)take(n * a->dv * 8);
    P.pNe = (uint64_t*)take(n * a->dv * 8);
    P.pR = (int32_t*)take(n * 4);
    P.pNR = (int32_t*)take(n * a->dv * 4);
    P.pSt = (int32_t*)take(n * 4);
  }
  P.q = a->q;
  P.k = a->k;
  P.v = a->v;
  P.rows = a->rows;
  P.d = a->d;
  P.dv = a->dv;
  int dl = ceil_log2(a->d);
  P.W = (61 - dl) / 2 > 28 ? 28 : (61 - dl) / 2;
  P.am = am;
  P.ae = ae;
  P.fp32 = a->fp32_out ? 1 : 0;
  P.kind = a->mask_kind;
  P.row_ptr = a->row_ptr;
  P.key_idx = a->key_idx;
  P.kv_base = a->kv_base;
  P.kv_len = a->kv_len;
  P.page_table = a->page_table;
  P.seq_lens = a->seq_lens;
  P.page_size = a->page_size;
  P.max_pages = a->max_pages;
  P.hq = a->q_heads;
  P.hkv = a->kv_heads;
  P.group = a->kv_heads > 0 ? a->q_heads / a->kv_heads : 1;
  P.splits = a->splits;
  P.key_log2 = ceil_log2(a->max_row_keys < 2 ? 2 : a->max_row_keys);
  P.FZ = 61 - P.key_log2;
  P.out = a->out;
  P.flags = a->flags;
  P.stats = a->stats ? (unsigned long long*)a->stats : stats;
  // what must start at zero: the tier-3 work-list counter (and the internal counters)
  cudaError_t e = cudaMemsetAsync(P.t3_count, 0, sizeof(int), st);
  if (e == cudaSuccess && !a->stats) e = cudaMemsetAsync(stats, 0, EA_STATS_LEN * 8, st);
  if (e == cudaSuccess) e = launch_simt(P, st);
  if (e == cudaSuccess) e = launch_tier3(P, (int)(a->rows < 2 * sms ? a->rows : 2 * sms), st);
  if (e != cudaSuccess) {
    g_err = std::string("ea_attention_cuda_noalloc: ") + cudaGetErrorString(e);
    return -4;
  }
  return 0;
}
