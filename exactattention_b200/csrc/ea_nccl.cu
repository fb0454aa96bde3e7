// The KV-shard merge of row partials over an NCCL communicator, as one C entry point: the C form of
// exactattention_b200/dist.py's merge for callers that hold an ncclComm_t (a C / C++ server).
//
//   1. all-reduce MAX of R, status and NR (R and NR into copies: the rescale needs both the local
//      and the global exponents)
//   2. every rank re-expresses its sums at the global exponents (ea_partials_rescale_cuda)
//   3. all-reduce SUM of Z, Zerr, N, Nerr
// MAX and SUM on integers are associative and commutative, so any ring or tree gives the same bits.
// NCCL is loaded at run time (libnccl.so.2; an already loaded copy is preferred, so the caller's
// communicator and these calls use the same library): the library does not link against NCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "../../include/exactattn_cuda.h"

namespace {

struct NcclApi {
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  bool ok = false;
};

const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    api.all_reduce = (decltype(&ncclAllReduce))dlsym(h, "ncclAllReduce");
    api.group_start = (decltype(&ncclGroupStart))dlsym(h, "ncclGroupStart");
    api.group_end = (decltype(&ncclGroupEnd))dlsym(h, "ncclGroupEnd");
    api.ok = api.all_reduce && api.group_start && api.group_end;
  });
  return api;
}

// per-device scratch for the global exponents (grow only); calls on one device share it, so a
// caller orders its merges on one device (one stream, or events between streams)
struct MergeScratch {
  int32_t* buf = nullptr;
  size_t n = 0;
};
std::mutex g_mu;
MergeScratch g_scratch[64];

int32_t* scratch(size_t n) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  MergeScratch& s = g_scratch[dev];
  if (s.n < n) {
    if (s.buf) cudaFree(s.buf);
    s.buf = nullptr;
    s.n = 0;
    if (cudaMalloc(&s.buf, n * sizeof(int32_t)) != cudaSuccess) return nullptr;
    s.n = n;
  }
  return s.buf;
}

}  // namespace

namespace ea {
// frees the merge scratch of every device (ea_cuda_release)
void nccl_release_scratch() {
  std::lock_guard<std::mutex> lk(g_mu);
  int cur = 0;
  cudaGetDevice(&cur);
  for (int d = 0; d < 64; ++d) {
    MergeScratch& s = g_scratch[d];
    if (!s.buf) continue;
    cudaSetDevice(d);
    cudaFree(s.buf);
    s.buf = nullptr;
    s.n = 0;
  }
  cudaSetDevice(cur);
}
}  // namespace ea

extern "C" int ea_merge_partials_nccl(const ea_partials_t* parts, int64_t rows, int dv, void* nccl_comm,
                                      void* stream) {
  if (!parts || rows < 0 || dv <= 0 || !nccl_comm) return -1;
  const NcclApi& api = nccl_api();
  if (!api.ok) return -7;
  ncclComm_t comm = (ncclComm_t)nccl_comm;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t nr = (size_t)rows, nc = (size_t)rows * (size_t)dv;
  int32_t* g = scratch(nr + nc);
  if (!g && rows > 0) return -4;
  int32_t* Rg = g;
  int32_t* NRg = g + nr;
  // 1. global maxima (every rank takes the same collective steps, also for rows == 0)
  if (rows > 0) {
    if (cudaMemcpyAsync(Rg, parts->R, nr * sizeof(int32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess) return -4;
    if (cudaMemcpyAsync(NRg, parts->NR, nc * sizeof(int32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess) return -4;
  }
  ncclResult_t r = api.group_start();
  if (r == ncclSuccess) r = api.all_reduce(Rg, Rg, nr, ncclInt32, ncclMax, comm, st);
  if (r == ncclSuccess) r = api.all_reduce(NRg, NRg, nc, ncclInt32, ncclMax, comm, st);
  if (r == ncclSuccess) r = api.all_reduce(parts->status, parts->status, nr, ncclInt32, ncclMax, comm, st);
  const ncclResult_t re = api.group_end();
  if (r != ncclSuccess || re != ncclSuccess) return -8;
  // 2. the local sums at the global exponents
  int rc = ea_partials_rescale_cuda(parts, Rg, NRg, rows, dv, stream);
  if (rc) return rc;
  // 3. sums
  r = api.group_start();
  if (r == ncclSuccess) r = api.all_reduce(parts->Z, parts->Z, nr, ncclInt64, ncclSum, comm, st);
  if (r == ncclSuccess) r = api.all_reduce(parts->Zerr, parts->Zerr, nr, ncclInt64, ncclSum, comm, st);
  if (r == ncclSuccess) r = api.all_reduce(parts->N, parts->N, nc, ncclInt64, ncclSum, comm, st);
  if (r == ncclSuccess) r = api.all_reduce(parts->Nerr, parts->Nerr, nc, ncclInt64, ncclSum, comm, st);
  const ncclResult_t re2 = api.group_end();
  if (r != ncclSuccess || re2 != ncclSuccess) return -8;
  // the partials now hold the merged exponents (the rescale wrote them) and sums
  return 0;
}
