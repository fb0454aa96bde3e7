// C ABI of libexactattn_cuda.so (declared in include/exactattn_cuda.h): argument checks,
// the per-device workspace, and the launch sequence tier 1 -> combine -> tier 3.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <deque>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/exactattn_cuda.h"
#include "ea_core.cuh"
#include "ea_wide.h"

namespace ea {
cudaError_t launch_simt(const Prob& P, cudaStream_t st);
cudaError_t launch_tier3(const Prob& P, int blocks, cudaStream_t st);
cudaError_t launch_tc_prefill(const Prob& P, const int32_t* block_rows, int64_t nblocks, cudaStream_t st);
cudaError_t launch_partials_rescale(const Prob& P, const int32_t* Rg, const int32_t* NRg, cudaStream_t st);
cudaError_t launch_partials_finalize(const Prob& P, cudaStream_t st);
cudaError_t launch_gathered_merge(const Prob& P, const void* g, int world, int64_t stride, int* wide_rows,
                                  int* wide_count, cudaStream_t st);
cudaError_t launch_combine(const Prob& P, cudaStream_t st);
cudaError_t launch_tc_decode(const Prob& P, const int32_t* seg_rows, int64_t nseg, int max_rows, cudaStream_t st);
cudaError_t launch_wide_rescale(const Prob& P, int n, const int64_t* gmax, cudaStream_t st);
cudaError_t launch_wide_finalize(const Prob& P, int n, const int64_t* gmax, cudaStream_t st);
cudaError_t launch_list_all_rows(const Prob& P, cudaStream_t st);
cudaError_t launch_fallback(const Prob& P, const FallbackBufs& F, int sms, cudaStream_t st);
size_t fallback_bytes(int dv);
void fallback_carve(void* base, int dv, FallbackBufs& F);
void nccl_release_scratch();  // ea_nccl.cu
}  // namespace ea

using namespace ea;

static_assert(EA_STATS_LEN == STAT_LEN, "the C ABI's stats length and the device counters agree");

namespace {

thread_local std::string g_err;

// the full counters of this thread's last host-pointer call (ea_last_host_stats)
thread_local int64_t g_last_host_stats[EA_STATS_LEN] = {0};

// test hooks (ea_set_test_hooks), copied into every launch's problem description
ea_test_hooks_t g_hooks = {0, 0, 0};

int fail_cuda(cudaError_t e, const char* where) {
  g_err = std::string(where) + ": " + cudaGetErrorString(e);
  return -4;
}

// Grow-only device buffers of one device. Each device has two: one for the device-pointer entry
// points (callers order their launches on one device) and one for the synchronous host-pointer
// entry points, whose calls host_mu serialises, so that concurrent host calls (the reference's C
// entry is reentrant) never share staging or partial buffers with work in flight.
struct Workspace {
  int device = -1;
  bool host = false;
  std::mutex host_mu;
  int sms = 148;
  unsigned long long* stats = nullptr;  // STAT_LEN
  int* t3_count = nullptr;
  int* t3_list = nullptr;
  int64_t t3_cap = 0;
  // the fallback tiers: tier 3's row list (capacity t3_cap, after the count in list3_blk) and
  // the fixed-size tier-2 / tier-3 buffers for fb_dv channels
  void* list3_blk = nullptr;
  void* fb = nullptr;
  int fb_dv = 0;
  FallbackBufs F{};
  void* part = nullptr;
  size_t part_bytes = 0;
  // staging for the host-pointer entry point, and the row lists it builds on the host (pinned)
  // and copies (device)
  void* stage = nullptr;
  size_t stage_bytes = 0;
  int32_t* lists_h = nullptr;
  size_t lists_h_bytes = 0;
  void* lists = nullptr;
  size_t lists_bytes = 0;
  cudaStream_t stream = nullptr;
  // a side stream and fork / join events for work that can overlap on one launch (the tree
  // mask's list part beside the tensor-core range part)
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

std::mutex g_mu;
std::deque<Workspace> g_ws;  // a deque: workspaces never move once made

// the current device's workspace (call with g_mu held)
Workspace* workspace(bool host = false) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  for (auto& w : g_ws)
    if (w.device == dev && w.host == host) return &w;
  unsigned long long* stats = nullptr;
  int* t3_count = nullptr;
  if (cudaMalloc(&stats, STAT_LEN * sizeof(unsigned long long)) != cudaSuccess) return nullptr;
  if (cudaMalloc(&t3_count, sizeof(int)) != cudaSuccess) {
    cudaFree(stats);
    return nullptr;
  }
  cudaMemset(stats, 0, STAT_LEN * sizeof(unsigned long long));
  Workspace& w = g_ws.emplace_back();
  w.device = dev;
  w.host = host;
  cudaDeviceGetAttribute(&w.sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaStreamCreateWithFlags(&w.side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&w.fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&w.join, cudaEventDisableTiming) != cudaSuccess)
    w.side = nullptr;  // (then the list part runs on the launch stream)
  w.stats = stats;
  w.t3_count = t3_count;
  return &w;
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// the split partial buffers as build_prob carves them: Z, Zerr, N, Nerr, R, NR, status
size_t part_bytes(int64_t rows, int splits, int dv) {
  if (splits <= 1) return 0;
  const size_t n = (size_t)rows * (size_t)splits;
  return 2 * align256(n * 8) + 2 * align256(n * dv * 8) + align256(n * 4) + align256(n * dv * 4) + align256(n * 4);
}

bool grow(void** p, size_t* cap, size_t need) {
  if (need <= *cap) return true;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  size_t n = need + need / 4;
  if (cudaMalloc(p, n) != cudaSuccess) return false;
  *cap = n;
  return true;
}

int reserve(Workspace* w, int64_t rows, int splits, int dv) {
  if (rows > w->t3_cap) {
    if (w->t3_list) cudaFree(w->t3_list);
    if (w->list3_blk) cudaFree(w->list3_blk);
    w->t3_list = nullptr;
    w->list3_blk = nullptr;
    w->t3_cap = 0;
    if (cudaMalloc(&w->t3_list, (size_t)rows * sizeof(int)) != cudaSuccess) return fail_cuda(cudaErrorMemoryAllocation, "t3_list");
    if (cudaMalloc(&w->list3_blk, 256 + (size_t)rows * sizeof(int)) != cudaSuccess)
      return fail_cuda(cudaErrorMemoryAllocation, "tier-3 list");
    w->t3_cap = rows;
    w->F.count3 = (int*)w->list3_blk;
    w->F.list3 = (int*)((char*)w->list3_blk + 256);
  }
  const int fdv = dv <= 32 ? 32 : dv <= 64 ? 64 : dv <= 128 ? 128 : 256;  // the fallback buffers' width
  if (dv <= 256 && fdv > w->fb_dv) {
    if (w->fb) cudaFree(w->fb);
    w->fb = nullptr;
    w->fb_dv = 0;
    if (cudaMalloc(&w->fb, fallback_bytes(fdv)) != cudaSuccess) return fail_cuda(cudaErrorMemoryAllocation, "fallback");
    w->fb_dv = fdv;
  }
  if (!grow(&w->part, &w->part_bytes, part_bytes(rows, splits, dv)))
    return fail_cuda(cudaErrorMemoryAllocation, "partials");
  return 0;
}

int window_bits(int d) {
  int dl = 0;
  while ((1 << dl) < d) ++dl;
  int W = (61 - dl) / 2;
  return W > 28 ? 28 : W;
}

int ceil_log2(int64_t n) {
  int k = 0;
  while (((int64_t)1 << k) < n) ++k;
  return k;
}

}  // namespace

extern "C" {

const char* ea_cuda_last_error(void) { return g_err.c_str(); }

int ea_reserve_workspace(int64_t rows, int splits, int dv) {
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace* w = workspace();
  if (!w) return fail_cuda(cudaGetLastError(), "workspace");
  // the tree-mask and decode paths keep split partials even at one split: reserve for two
  return reserve(w, rows, splits < 2 ? 2 : splits, dv);
}

void ea_cuda_release(void) {
  nccl_release_scratch();
  std::lock_guard<std::mutex> lk(g_mu);
  int cur = 0;
  cudaGetDevice(&cur);
  for (auto& w : g_ws) {
    cudaSetDevice(w.device);
    if (w.stats) cudaFree(w.stats);
    if (w.t3_count) cudaFree(w.t3_count);
    if (w.t3_list) cudaFree(w.t3_list);
    if (w.list3_blk) cudaFree(w.list3_blk);
    if (w.fb) cudaFree(w.fb);
    if (w.part) cudaFree(w.part);
    if (w.stage) cudaFree(w.stage);
    if (w.lists) cudaFree(w.lists);
    if (w.lists_h) cudaFreeHost(w.lists_h);
    if (w.stream) cudaStreamDestroy(w.stream);
    if (w.side) cudaStreamDestroy(w.side);
    if (w.fork) cudaEventDestroy(w.fork);
    if (w.join) cudaEventDestroy(w.join);
  }
  g_ws.clear();
  cudaSetDevice(cur);
}

// ---------------------------------------------------------------------------
// optional timing of the tier-1 kernel: CUDA events recorded on the launch stream around it
// ---------------------------------------------------------------------------
struct KernelTiming {
  bool on = false;
  std::vector<cudaEvent_t> ev;  // pairs (start, end)
  size_t used = 0;
};
static KernelTiming g_kt;

// A tier-1 launch records its start/end events when timing is on (events come from a pool that
// is created when timing is switched on, so nothing is allocated per launch).
struct TimedLaunch {
  cudaStream_t st;
  cudaEvent_t end = nullptr;
  explicit TimedLaunch(cudaStream_t s) : st(s) {
    if (g_kt.on && g_kt.used + 2 <= g_kt.ev.size()) {
      cudaEventRecord(g_kt.ev[g_kt.used], st);
      end = g_kt.ev[g_kt.used + 1];
      g_kt.used += 2;
    }
  }
  ~TimedLaunch() {
    if (end) cudaEventRecord(end, st);
  }
};

static int check_launch(const ea_launch_t* a) {
  if (!a || a->d <= 0 || a->d > 1024 || a->dv <= 0 || a->splits <= 0 || a->splits > 65535 || a->rows < 0) return -1;
  uint32_t ab;
  memcpy(&ab, &a->alpha, 4);
  int32_t am, ae;
  if (!decode_fp32(ab, am, ae)) return -3;
  if (a->mask_kind < EA_MASK_CSR || a->mask_kind > EA_MASK_HYBRID) return -9;
  if (a->mask_kind == EA_MASK_PAGED && (a->page_size <= 0 || a->q_heads <= 0 || a->kv_heads <= 0 ||
                                        a->q_heads % a->kv_heads != 0))
    return -9;
  return 0;
}

// The fallback buffers of workspace w carved for dv channels (reserve() sized them).
static FallbackBufs fallback_bufs(Workspace* w, int dv) {
  FallbackBufs F = w->F;
  fallback_carve(w->fb, dv, F);
  return F;
}

// Problem description from the launch arguments, with the workspace's split buffers when
// splits > 1.
static void build_prob(const ea_launch_t* a, Workspace* w, Prob& P) {
  uint32_t ab;
  memcpy(&ab, &a->alpha, 4);
  int32_t am, ae;
  decode_fp32(ab, am, ae);
  memset(&P, 0, sizeof(P));
  P.q = a->q;
  P.k = a->k;
  P.v = a->v;
  P.rows = a->rows;
  P.d = a->d;
  P.dv = a->dv;
  P.W = window_bits(a->d);
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
  P.krows = a->nkeys;
  P.hq = a->q_heads;
  P.hkv = a->kv_heads;
  P.group = a->kv_heads > 0 ? a->q_heads / a->kv_heads : 1;
  P.splits = a->splits;
  int64_t mk = a->max_row_keys < 2 ? 2 : a->max_row_keys;
  P.key_log2 = ceil_log2(mk);
  P.FZ = 61 - P.key_log2;
  P.out = a->out;
  P.flags = a->flags;
  P.stats = a->stats ? (unsigned long long*)a->stats : w->stats;
  P.t3_count = w->t3_count;
  P.t3_list = w->t3_list;
  P.tier = 1;
  P.force_stride = g_hooks.force_stride;
  P.force_tier = g_hooks.force_tier;
  P.wait_debug = g_hooks.wait_debug;
  if (a->splits > 1) {
    int64_t n = a->rows * (int64_t)a->splits;
    char* p = (char*)w->part;
    auto take = [&](size_t bytes) {
      char* r = p;
      p += (bytes + 255) & ~(size_t)255;
      return (void*)r;
    };
    P.pZ = (int64_t*)take(n * 8);
    P.pZe = (uint64_t*)take(n * 8);
    P.pN = (int64_t*)take(n * a->dv * 8);
    P.pNe = (uint64_t*)take(n * a->dv * 8);
    P.pR = (int32_t*)take(n * 4);
    P.pNR = (int32_t*)take(n * a->dv * 4);
    P.pSt = (int32_t*)take(n * 4);
  }
}

static bool tc_shape(const ea_launch_t* a) {
  return a->block_rows && a->nblocks > 0 && a->d == 128 && a->dv == 128 && ((uintptr_t)a->q & 15) == 0 &&
         ((uintptr_t)a->k & 15) == 0;
}

// RANGE masks with row blocks: the tensor-core prefill kernel (KV splits on its grid's y, merged
// by the split combine)
static bool tc_applicable(const ea_launch_t* a) {
  return a->mask_kind == EA_MASK_RANGE && tc_shape(a);
}

// A HYBRID mask (shared key range + per-row list: tree verification) with row blocks: the range
// part on the tensor cores and the list part on the CUDA cores, each exporting its partial into
// one of two split slots, merged and finalised by the split combine (the merge of split
// partials is exact, so this is the same as one pass over the row's keys).
static bool hybrid_tc_applicable(const ea_launch_t* a) {
  return a->mask_kind == EA_MASK_HYBRID && tc_shape(a);
}

// Decode shapes: a few rows per key sequence (a GQA group). PAGED masks form their segments from
// the layout (sequence, kv head); RANGE masks need the caller's segment table.
static bool decode_applicable(const ea_launch_t* a) {
  if (a->d != 128 || a->dv != 128 || ((uintptr_t)a->q & 15) || ((uintptr_t)a->k & 15) || ((uintptr_t)a->v & 15))
    return false;
  if (a->mask_kind == EA_MASK_RANGE) return a->seg_rows && a->nsegs > 0;
  if (a->mask_kind == EA_MASK_PAGED)
    return a->q_heads > 0 && a->kv_heads > 0 && a->q_heads / a->kv_heads <= 8 && a->rows % a->q_heads == 0;
  return false;
}

static int64_t decode_segments(const ea_launch_t* a) {
  return a->mask_kind == EA_MASK_PAGED ? (a->rows / a->q_heads) * a->kv_heads : a->nsegs;
}

// rows per decode segment: the GQA group of a paged layout; a segment table may fill all 8 slots
static int decode_max_rows(const ea_launch_t* a) {
  if (a->mask_kind == EA_MASK_PAGED) return a->q_heads / a->kv_heads;
  return a->seg_width >= 1 && a->seg_width <= 8 ? a->seg_width : 8;
}

// the decode kernel writes split partials for splits >= 1: carve the split buffers for at least 2
static int decode_prob(const ea_launch_t* a, Workspace* w, Prob& P) {
  ea_launch_t a2 = *a;
  a2.splits = a->splits < 2 ? 2 : a->splits;
  int rc = reserve(w, a2.rows, a2.splits, a2.dv);
  if (rc) return rc;
  build_prob(&a2, w, P);
  P.splits = a->splits;
  return 0;
}

static int launch_decode_tc(const ea_launch_t* a, Workspace* w, cudaStream_t st) {
  Prob P;
  int rc = decode_prob(a, w, P);
  if (rc) return rc;
  cudaError_t e = cudaMemsetAsync(w->t3_count, 0, sizeof(int), st);
  if (e != cudaSuccess) return fail_cuda(e, "memset");
  const int32_t* seg = a->mask_kind == EA_MASK_RANGE ? a->seg_rows : nullptr;
  {
    TimedLaunch tl(st);
    e = launch_tc_decode(P, seg, decode_segments(a), decode_max_rows(a), st);
  }
  if (e != cudaSuccess) return fail_cuda(e, "tier-1 decode launch");
  e = launch_combine(P, st);
  if (e != cudaSuccess) return fail_cuda(e, "combine");
  e = launch_fallback(P, fallback_bufs(w, a->dv), w->sms, st);
  if (e != cudaSuccess) return fail_cuda(e, "fallback tiers");
  return 0;
}

static void export_to_split(Prob& X, const Prob& P, int s) {
  const int64_t o = (int64_t)s * P.rows;
  X.splits = 1;
  X.export_partials = 1;
  X.xR = P.pR + o;
  X.xZ = P.pZ + o;
  X.xZe = P.pZe + o;
  X.xSt = P.pSt + o;
  X.xNR = P.pNR + o * P.dv;
  X.xN = P.pN + o * P.dv;
  X.xNe = P.pNe + o * P.dv;
}

// The range part runs in a0->splits KV splits on the tensor cores (split slots 0 .. S - 1), the
// per-row lists on the CUDA cores (slot S); one exact combine merges the S + 1 slots.
static int launch_hybrid_tc(const ea_launch_t* a0, Workspace* w, cudaStream_t st) {
  const int S = a0->splits;
  ea_launch_t a = *a0;
  a.splits = S + 1;
  int rc = reserve(w, a.rows, S + 1, a.dv);
  if (rc) return rc;
  Prob P;
  build_prob(&a, w, P);
  cudaError_t e = cudaMemsetAsync(w->t3_count, 0, sizeof(int), st);
  if (e != cudaSuccess) return fail_cuda(e, "memset");
  Prob P0 = P;
  P0.kind = MASK_RANGE;
  if (S == 1)
    export_to_split(P0, P, 0);
  else
    P0.splits = S;  // the kernel's grid.y: split y writes split slot y
  // the list part (its own split slot) runs beside the range part, on the side stream
  Prob P1 = P;
  P1.kind = MASK_CSR;
  export_to_split(P1, P, S);
  cudaStream_t ls = st;
  if (w->side && cudaEventRecord(w->fork, st) == cudaSuccess && cudaStreamWaitEvent(w->side, w->fork, 0) == cudaSuccess)
    ls = w->side;
  e = launch_simt(P1, ls);
  if (e != cudaSuccess) return fail_cuda(e, "tier-1 list launch");
  if (ls != st && ((e = cudaEventRecord(w->join, ls)) != cudaSuccess)) return fail_cuda(e, "join");
  {
    TimedLaunch tl(st);
    e = launch_tc_prefill(P0, a.block_rows, a.nblocks, st);
  }
  if (e != cudaSuccess) return fail_cuda(e, "tier-1 range launch");
  if (ls != st && (e = cudaStreamWaitEvent(st, w->join, 0)) != cudaSuccess) return fail_cuda(e, "join");
  e = launch_combine(P, st);
  if (e != cudaSuccess) return fail_cuda(e, "combine");
  e = launch_fallback(P, fallback_bufs(w, a.dv), w->sms, st);
  if (e != cudaSuccess) return fail_cuda(e, "fallback tiers");
  return 0;
}

// More than 256 value channels (beyond what the tier-1 and tier-2 kernels keep per thread): every
// row goes straight to the wide tier 3, which loops over channel blocks of any width.
static int launch_wide_all(const ea_launch_t* a0, Workspace* w, cudaStream_t st) {
  ea_launch_t a = *a0;
  a.splits = 1;
  int rc = reserve(w, a.rows, 1, a.dv);
  if (rc) return rc;
  Prob P;
  build_prob(&a, w, P);
  cudaError_t e = launch_list_all_rows(P, st);
  if (e != cudaSuccess) return fail_cuda(e, "row list");
  int blocks = (int)(a.rows < 2 * w->sms ? a.rows : 2 * w->sms);
  e = launch_tier3(P, blocks, st);
  if (e != cudaSuccess) return fail_cuda(e, "tier-3 launch");
  return 0;
}

// the launch sequence of one problem on workspace w (g_mu held)
static int launch_on(const ea_launch_t* a, Workspace* w, cudaStream_t st) {
  int rc;
  if (a->dv > 256) return launch_wide_all(a, w, st);
  if (hybrid_tc_applicable(a)) return launch_hybrid_tc(a, w, st);
  if (decode_applicable(a)) return launch_decode_tc(a, w, st);
  rc = reserve(w, a->rows, a->splits, a->dv);
  if (rc) return rc;
  Prob P;
  build_prob(a, w, P);
  cudaError_t e = cudaMemsetAsync(w->t3_count, 0, sizeof(int), st);
  if (e != cudaSuccess) return fail_cuda(e, "memset");
  const bool tc = tc_applicable(a);
  {
    TimedLaunch tl(st);
    e = tc ? launch_tc_prefill(P, a->block_rows, a->nblocks, st) : launch_simt(P, st);
  }
  if (e == cudaSuccess && tc && a->splits > 1) e = launch_combine(P, st);
  if (e != cudaSuccess) return fail_cuda(e, "tier-1 launch");
  e = launch_fallback(P, fallback_bufs(w, a->dv), w->sms, st);
  if (e != cudaSuccess) return fail_cuda(e, "fallback tiers");
  return 0;
}

int ea_launch_cuda(const ea_launch_t* a, void* stream) {
  int rc = check_launch(a);
  if (rc) return rc;
  if (a->rows == 0) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace* w = workspace();
  if (!w) return fail_cuda(cudaGetLastError(), "workspace");
  return launch_on(a, w, (cudaStream_t)stream);
}

// The host-pointer entry points' workspace with its call lock taken: staging grown to `bytes`
// and a library stream. Returns nullptr after recording the error.
static Workspace* host_workspace(size_t bytes, std::unique_lock<std::mutex>& call) {
  Workspace* w;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    w = workspace(true);
    if (!w) {
      fail_cuda(cudaGetLastError(), "workspace");
      return nullptr;
    }
  }
  call = std::unique_lock<std::mutex>(w->host_mu);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!grow(&w->stage, &w->stage_bytes, bytes)) {
    fail_cuda(cudaErrorMemoryAllocation, "staging");
    return nullptr;
  }
  if (!w->stream && cudaStreamCreateWithFlags(&w->stream, cudaStreamNonBlocking) != cudaSuccess) {
    fail_cuda(cudaGetLastError(), "stream");
    return nullptr;
  }
  return w;
}

// ea_launch_cuda on the host-pointer workspace (its call lock held)
static int launch_host(const ea_launch_t* a, Workspace* w) {
  int rc = check_launch(a);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  return launch_on(a, w, w->stream);
}

static void set_export(Prob& P, const ea_partials_t* x) {
  P.export_partials = 1;
  P.xR = x->R;
  P.xZ = x->Z;
  P.xZe = (uint64_t*)x->Zerr;
  P.xSt = x->status;
  P.xNR = x->NR;
  P.xN = x->N;
  P.xNe = (uint64_t*)x->Nerr;
}

int ea_partials_cuda(const ea_launch_t* a, const ea_partials_t* x, void* stream) {
  int rc = check_launch(a);
  if (rc) return rc;
  if (!x || a->dv > 256) return -1;
  if (a->rows == 0) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace* w = workspace();
  if (!w) return fail_cuda(cudaGetLastError(), "workspace");
  cudaStream_t st = (cudaStream_t)stream;
  Prob P;
  if (decode_applicable(a)) {
    rc = decode_prob(a, w, P);
    if (rc) return rc;
    set_export(P, x);
    const int32_t* seg = a->mask_kind == EA_MASK_RANGE ? a->seg_rows : nullptr;
    cudaError_t e;
    {
      TimedLaunch tl(st);
      e = launch_tc_decode(P, seg, decode_segments(a), decode_max_rows(a), st);
    }
    if (e == cudaSuccess) e = launch_combine(P, st);
    return e == cudaSuccess ? 0 : fail_cuda(e, "partials decode launch");
  }
  rc = reserve(w, a->rows, a->splits, a->dv);
  if (rc) return rc;
  build_prob(a, w, P);
  set_export(P, x);
  cudaError_t e;
  const bool tc = tc_applicable(a);
  {
    TimedLaunch tl(st);
    e = tc ? launch_tc_prefill(P, a->block_rows, a->nblocks, st) : launch_simt(P, st);
  }
  if (e == cudaSuccess && tc && a->splits > 1) e = launch_combine(P, st);  // split partials -> export
  if (e != cudaSuccess) return fail_cuda(e, "partials launch");
  return 0;
}

int ea_partials_rescale_cuda(const ea_partials_t* x, const int32_t* R_global, const int32_t* NR_global,
                             int64_t rows, int dv, void* stream) {
  if (!x || rows < 0 || dv <= 0) return -1;
  if (rows == 0) return 0;
  Prob P;
  memset(&P, 0, sizeof(P));
  P.rows = rows;
  P.dv = dv;
  set_export(P, x);
  cudaError_t e = launch_partials_rescale(P, R_global, NR_global, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : fail_cuda(e, "rescale");
}

int ea_partials_finalize_cuda(const ea_partials_t* x, int64_t rows, int dv, int64_t max_row_keys, int fp32_out,
                              void* out, uint8_t* flags, int64_t* stats, void* stream) {
  if (!x || rows < 0 || dv <= 0 || !out || !flags) return -1;
  if (rows == 0) return 0;
  Workspace* w;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    w = workspace();
    if (!w) return fail_cuda(cudaGetLastError(), "workspace");
  }
  Prob P;
  memset(&P, 0, sizeof(P));
  P.rows = rows;
  P.dv = dv;
  P.fp32 = fp32_out ? 1 : 0;
  P.key_log2 = ceil_log2(max_row_keys < 2 ? 2 : max_row_keys);
  P.FZ = 61 - P.key_log2;
  P.out = out;
  P.flags = flags;
  P.stats = stats ? (unsigned long long*)stats : w->stats;
  set_export(P, x);
  cudaError_t e = launch_partials_finalize(P, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : fail_cuda(e, "finalize");
}

int ea_partials_merge_gathered_cuda(const void* gathered, int world, int64_t rows, int dv, int64_t max_row_keys,
                                    int fp32_out, void* out, uint8_t* flags, int32_t* wide_rows, int32_t* wide_count,
                                    int64_t* stats, void* stream) {
  if (!gathered || world <= 0 || rows < 0 || dv <= 0 || dv > 256 || !out || !flags || !wide_rows || !wide_count)
    return -1;
  if (rows == 0) return 0;
  Workspace* w;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    w = workspace();
    if (!w) return fail_cuda(cudaGetLastError(), "workspace");
  }
  Prob P;
  memset(&P, 0, sizeof(P));
  P.rows = rows;
  P.dv = dv;
  P.fp32 = fp32_out ? 1 : 0;
  P.key_log2 = ceil_log2(max_row_keys < 2 ? 2 : max_row_keys);
  P.FZ = 61 - P.key_log2;
  P.out = out;
  P.flags = flags;
  P.stats = stats ? (unsigned long long*)stats : w->stats;
  const int64_t stride = (int64_t)EA_PARTIALS_FLAT_BYTES(rows, dv);
  cudaError_t e = launch_gathered_merge(P, gathered, world, stride, wide_rows, wide_count, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : fail_cuda(e, "gathered merge");
}

// Rows grouped by kv_base: `order` lists the rows group by group (increasing kv_base, a group's
// rows in input order), group g being order[gstart[g] .. gstart[g + 1]). Rows already in
// non-decreasing kv_base order (the usual layout) take one pass; others one stable sort.
static void group_rows(const int64_t* kv_base, int64_t rows, std::vector<int32_t>& order,
                       std::vector<int64_t>& gstart) {
  order.resize((size_t)rows);
  for (int64_t i = 0; i < rows; ++i) order[i] = (int32_t)i;
  bool sorted = true;
  for (int64_t i = 1; i < rows && sorted; ++i) sorted = kv_base[i] >= kv_base[i - 1];
  if (!sorted)
    std::stable_sort(order.begin(), order.end(), [&](int32_t x, int32_t y) { return kv_base[x] < kv_base[y]; });
  gstart.clear();
  for (int64_t i = 0; i < rows; ++i)
    if (i == 0 || kv_base[order[i]] != kv_base[order[i - 1]]) gstart.push_back(i);
  gstart.push_back(rows);
}

// Rows [r0, r1) by decreasing kv_len, ties in their current order: a non-increasing run stays, a
// strictly increasing one (causal rows) is reversed, anything else is stably sorted.
static void order_by_len_desc(const int64_t* kv_len, int32_t* r0, int32_t* r1) {
  bool noninc = true, inc = true;
  for (int32_t* p = r0 + 1; p < r1; ++p) {
    noninc = noninc && kv_len[p[0]] <= kv_len[p[-1]];
    inc = inc && kv_len[p[0]] > kv_len[p[-1]];
  }
  if (noninc) return;
  if (inc) {
    std::reverse(r0, r1);
    return;
  }
  std::stable_sort(r0, r1, [&](int32_t x, int32_t y) { return kv_len[x] > kv_len[y]; });
}

// -5 when a bounded wait of a tensor-core kernel gave up during the call (a stalled GPU): the
// affected rows were recomputed by the later tiers, so out and flags are complete and exact.
static int wait_status(const int64_t* hs) {
  memcpy(g_last_host_stats, hs, sizeof(g_last_host_stats));
  if (hs[STAT_WAIT_EXPIRED] == 0) return 0;
  g_err = std::to_string(hs[STAT_WAIT_EXPIRED]) +
          " CTA(s) of a tensor-core kernel gave up a bounded wait; their rows were recomputed by the "
          "wide tier and the outputs are exact";
  return -5;
}

// KV splits the host entries choose for the tensor-core kernels when the caller leaves the
// schedule to the library (the reference's C entry takes `splits` for its CPU threads; the bits
// never depend on it): prefill a split per block unless the blocks are too few to fill the GPU;
// decode enough splits for about eight CTAs per SM, each at least 1024 keys.
static int auto_splits(bool decode, int64_t units, int64_t maxlen, int sms) {
  if (units <= 0) return 1;
  int64_t sp;
  if (decode) {
    sp = (8 * (int64_t)sms + units - 1) / units;
    sp = std::min<int64_t>(sp, std::max<int64_t>(1, maxlen / 1024));
  } else {
    if (units >= sms) return 1;
    sp = (sms + units - 1) / units;
    sp = std::min<int64_t>(sp, std::max<int64_t>(1, maxlen / 512));
  }
  return (int)std::max<int64_t>(1, std::min<int64_t>(sp, 64));
}

// Copies host inputs to the workspace, runs ea_launch_cuda, copies the results back. The mask:
// (row_ptr, key_idx) CSR; (kv_base, kv_len) ranges; both: HYBRID (the range, then the list);
// neither: every key. auto_sched: the library picks the KV splits of the tensor-core kernels.
static int run_host(const uint16_t* q, int64_t rows, int d, const uint16_t* k, const uint16_t* v, int64_t nkeys,
                    int dv, float alpha, const int64_t* row_ptr, const int64_t* key_idx, const int64_t* kv_base_h,
                    const int64_t* kv_len_h, int64_t maxn, int fp32_out, int splits, void* out, uint8_t* flags,
                    int64_t* stats, bool auto_sched = false) {
  int64_t total = row_ptr ? row_ptr[rows] : 0;
  std::vector<int64_t> kb, kl;
  if (!row_ptr && !kv_len_h) {  // every key: one range shared by all rows
    kb.assign(rows, 0);
    kl.assign(rows, nkeys);
    kv_base_h = kb.data();
    kv_len_h = kl.data();
  }
  const bool hybrid = row_ptr && kv_len_h;
  const size_t osz = fp32_out ? 4 : 2;
  // staging layout: q | k | v | mask | out | flags | stats; the copies start before the host
  // builds the row lists (blocks / segments) of a range mask
  size_t off = 0;
  auto slot = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~(size_t)255;
    return o;
  };
  size_t oq = slot((size_t)rows * d * 2), ok = slot((size_t)nkeys * d * 2), ov = slot((size_t)nkeys * dv * 2);
  size_t orp = slot((size_t)(rows + 1) * 8), oki = slot((size_t)(row_ptr ? total : 0) * 8);
  size_t okb = slot((size_t)(kv_len_h ? rows : 0) * 8), okl = slot((size_t)(kv_len_h ? rows : 0) * 8);
  size_t oo = slot((size_t)rows * dv * osz), of = slot((size_t)rows), os = slot(EA_STATS_LEN * 8);

  std::unique_lock<std::mutex> call;
  Workspace* w = host_workspace(off, call);
  if (!w) return -4;
  char* base = (char*)w->stage;
  cudaStream_t st = w->stream;
  cudaError_t e;
  // an error after the first copy waits for the copies in flight before the call returns
  auto fail = [&](cudaError_t err, const char* where) {
    cudaStreamSynchronize(st);
    return fail_cuda(err, where);
  };
#define EA_CPY(dst, src, n)                                                    \
  if ((n) > 0) {                                                              \
    e = cudaMemcpyAsync(base + (dst), (src), (n), cudaMemcpyHostToDevice, st); \
    if (e != cudaSuccess) return fail(e, "h2d");                              \
  }
  EA_CPY(oq, q, (size_t)rows * d * 2);
  EA_CPY(ok, k, (size_t)nkeys * d * 2);
  EA_CPY(ov, v, (size_t)nkeys * dv * 2);
  if (row_ptr) {
    EA_CPY(orp, row_ptr, (size_t)(rows + 1) * 8);
    EA_CPY(oki, key_idx, (size_t)total * 8);
  }
  if (kv_len_h) {
    EA_CPY(okb, kv_base_h, (size_t)rows * 8);
    EA_CPY(okl, kv_len_h, (size_t)rows * 8);
  }
#undef EA_CPY
  // Range masks at d = dv = 128: rows sharing kv_base either form decode segments (at most 8 rows
  // per key range: the decode kernel) or 128-row blocks, longest first (the prefill kernel),
  // built while the copies above run. HYBRID masks take blocks (their range part).
  std::vector<int32_t> blocks, segs;
  bool decode = false;
  int seg_width = 8;
  int64_t range_max = 0;
  if (kv_len_h && d == 128 && dv == 128 && rows < (1ll << 31)) {
    for (int64_t r = 0; r < rows; ++r) range_max = std::max(range_max, kv_len_h[r]);
    std::vector<int32_t> order;
    std::vector<int64_t> gstart;
    group_rows(kv_base_h, rows, order, gstart);
    const int64_t ng = (int64_t)gstart.size() - 1;
    int64_t gmax = 0;
    for (int64_t g = 0; g < ng; ++g) gmax = std::max(gmax, gstart[g + 1] - gstart[g]);
    decode = gmax <= 8 && !hybrid;
    if (decode) {
      segs.assign((size_t)ng * 8, -1);
      for (int64_t g = 0; g < ng; ++g)
        for (int64_t u = gstart[g]; u < gstart[g + 1]; ++u) segs[(size_t)(8 * g + u - gstart[g])] = order[u];
      seg_width = (int)gmax;
    } else {
      // rows of a group by decreasing kv_len, cut into 128-row blocks; blocks by decreasing
      // length of their first (longest) row
      std::vector<int64_t> bst;  // first position in `order` of each block
      for (int64_t g = 0; g < ng; ++g) {
        order_by_len_desc(kv_len_h, order.data() + gstart[g], order.data() + gstart[g + 1]);
        for (int64_t c = gstart[g]; c < gstart[g + 1]; c += 128) bst.push_back(c);
      }
      std::stable_sort(bst.begin(), bst.end(),
                       [&](int64_t x, int64_t y) { return kv_len_h[order[x]] > kv_len_h[order[y]]; });
      blocks.assign(bst.size() * 128, -1);
      for (size_t i = 0; i < bst.size(); ++i) {
        const int64_t c = bst[i];
        const int64_t gend = gstart[std::upper_bound(gstart.begin(), gstart.end(), c) - gstart.begin()];
        std::copy(order.begin() + c, order.begin() + std::min(c + 128, gend), blocks.begin() + 128 * i);
      }
    }
  }
  const size_t nlist = blocks.size() + segs.size();
  if (nlist) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (w->lists_h_bytes < nlist * 4) {
      if (w->lists_h) cudaFreeHost(w->lists_h);
      w->lists_h = nullptr;
      w->lists_h_bytes = 0;
      if (cudaHostAlloc((void**)&w->lists_h, nlist * 4, cudaHostAllocDefault) != cudaSuccess)
        return fail(cudaErrorMemoryAllocation, "row lists");
      w->lists_h_bytes = nlist * 4;
    }
    if (!grow(&w->lists, &w->lists_bytes, nlist * 4)) return fail(cudaErrorMemoryAllocation, "row lists");
  }
  // the previous call's copy out of lists_h ended with its stream synchronisation
  int32_t* lists_d = (int32_t*)w->lists;
  if (nlist) {
    std::copy(blocks.begin(), blocks.end(), w->lists_h);
    std::copy(segs.begin(), segs.end(), w->lists_h + blocks.size());
    e = cudaMemcpyAsync(lists_d, w->lists_h, nlist * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return fail(e, "h2d");
  }
  e = cudaMemsetAsync(base + os, 0, EA_STATS_LEN * 8, st);
  if (e != cudaSuccess) return fail(e, "memset");

  ea_launch_t a;
  memset(&a, 0, sizeof(a));
  a.q = (const uint16_t*)(base + oq);
  a.rows = rows;
  a.d = d;
  a.k = (const uint16_t*)(base + ok);
  a.v = (const uint16_t*)(base + ov);
  a.nkeys = nkeys;
  a.dv = dv;
  a.alpha = alpha;
  a.mask_kind = hybrid ? EA_MASK_HYBRID : row_ptr ? EA_MASK_CSR : EA_MASK_RANGE;
  a.row_ptr = (const int64_t*)(base + orp);
  a.key_idx = (const int64_t*)(base + oki);
  a.kv_base = (const int64_t*)(base + okb);
  a.kv_len = (const int64_t*)(base + okl);
  a.max_row_keys = maxn;
  a.fp32_out = fp32_out;
  a.splits = splits;
  a.out = base + oo;
  a.flags = (uint8_t*)(base + of);
  a.stats = (int64_t*)(base + os);
  a.block_rows = blocks.empty() ? nullptr : lists_d;
  a.nblocks = (int64_t)(blocks.size() / 128);
  a.seg_rows = segs.empty() ? nullptr : lists_d + blocks.size();
  a.nsegs = (int64_t)(segs.size() / 8);
  a.seg_width = seg_width;
  if (auto_sched && (a.nblocks > 0 || a.nsegs > 0))
    a.splits = auto_splits(a.nsegs > 0, a.nsegs > 0 ? a.nsegs : a.nblocks, range_max, w->sms);
  int rc = launch_host(&a, w);
  if (rc) {
    cudaStreamSynchronize(st);
    return rc;
  }
  int64_t hs[EA_STATS_LEN];
  if ((e = cudaMemcpyAsync(out, base + oo, (size_t)rows * dv * osz, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
      (e = cudaMemcpyAsync(flags, base + of, (size_t)rows, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
      (e = cudaMemcpyAsync(hs, base + os, sizeof(hs), cudaMemcpyDeviceToHost, st)) != cudaSuccess)
    return fail(e, "d2h");
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return fail_cuda(e, "sync");
  if (stats) {
    stats[0] += hs[STAT_SCORE_EXACT];
    stats[1] += hs[STAT_WEIGHT_WIDE];
    stats[2] += hs[STAT_TIER1_UNCERT];
  }
  return wait_status(hs);
}

int ea_attention_cuda(const uint16_t* q, int64_t rows, int d, const uint16_t* k, const uint16_t* v,
                      int64_t nkeys, int dv, float alpha, const int64_t* row_ptr, const int64_t* key_idx,
                      int fp32_out, int acc_bits, int tile, int splits, uint64_t order_seed, int nthreads,
                      void* out, uint8_t* flags, int64_t* stats) {
  (void)order_seed;
  (void)nthreads;
  if (d <= 0 || d > 1024 || dv <= 0 || tile <= 0 || splits <= 0 || splits > 65535) return -1;
  if (acc_bits != 64 && acc_bits != 128) return -2;
  uint32_t ab;
  memcpy(&ab, &alpha, 4);
  int32_t am, ae;
  if (!decode_fp32(ab, am, ae)) return -3;
  if (rows <= 0) return 0;
  int64_t maxn = 1;
  if (!row_ptr) {
    return run_host(q, rows, d, k, v, nkeys, dv, alpha, nullptr, nullptr, nullptr, nullptr, std::max<int64_t>(1, nkeys),
                    fp32_out, splits, out, flags, stats, true);
  }
  for (int64_t r = 0; r < rows; ++r) maxn = std::max(maxn, row_ptr[r + 1] - row_ptr[r]);
  // The reference's callers pass CSR lists that are mostly runs of consecutive keys (causal and
  // prefix masks, tree masks as prefix + ancestors): each row's leading ascending run becomes a
  // key range, the rest stays a list. All runs: a RANGE mask; mostly runs (at d = dv = 128): a
  // HYBRID mask (the ranges on the tensor cores, the lists on the CUDA cores, merged exactly).
  // The same keys in a different layout give the same bits.
  std::vector<int64_t> kb((size_t)rows), kl((size_t)rows);
  int64_t tail = 0;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t p0 = row_ptr[r], p1 = row_ptr[r + 1];
    int64_t m = 0;
    kb[r] = p1 > p0 ? key_idx[p0] : 0;
    if (p1 > p0)
      for (m = 1; p0 + m < p1 && key_idx[p0 + m] == kb[r] + m;) ++m;
    kl[r] = m;
    tail += (p1 - p0) - m;
  }
  const int64_t total = row_ptr[rows] - row_ptr[0];
  if (tail == 0)
    return run_host(q, rows, d, k, v, nkeys, dv, alpha, nullptr, nullptr, kb.data(), kl.data(), maxn, fp32_out, splits,
                    out, flags, stats, true);
  if (d == 128 && dv == 128 && 4 * tail <= total) {
    std::vector<int64_t> trp((size_t)rows + 1), tki;
    tki.reserve((size_t)tail);
    for (int64_t r = 0; r < rows; ++r) {
      trp[r] = (int64_t)tki.size();
      tki.insert(tki.end(), key_idx + row_ptr[r] + kl[r], key_idx + row_ptr[r + 1]);
    }
    trp[rows] = (int64_t)tki.size();
    return run_host(q, rows, d, k, v, nkeys, dv, alpha, trp.data(), tki.data(), kb.data(), kl.data(), maxn, fp32_out,
                    splits, out, flags, stats, true);
  }
  return run_host(q, rows, d, k, v, nkeys, dv, alpha, row_ptr, key_idx, nullptr, nullptr, maxn, fp32_out, splits, out,
                  flags, stats, true);
}

int ea_attention_cuda_ranges(const uint16_t* q, int64_t rows, int d, const uint16_t* k, const uint16_t* v,
                             int64_t nkeys, int dv, float alpha, const int64_t* kv_base, const int64_t* kv_len,
                             int64_t max_row_keys, int fp32_out, int splits, void* out, uint8_t* flags,
                             int64_t* stats) {
  if (d <= 0 || d > 1024 || dv <= 0 || splits <= 0 || splits > 65535 || !kv_base || !kv_len) return -1;
  uint32_t ab;
  memcpy(&ab, &alpha, 4);
  int32_t am, ae;
  if (!decode_fp32(ab, am, ae)) return -3;
  if (rows <= 0) return 0;
  return run_host(q, rows, d, k, v, nkeys, dv, alpha, nullptr, nullptr, kv_base, kv_len,
                  max_row_keys < 1 ? 1 : max_row_keys, fp32_out, splits, out, flags, stats);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// ea_round_ratio_cuda: the reference's rounding export, evaluated by the device helper
// ---------------------------------------------------------------------------
namespace {
__global__ void round_ratio_kernel(uint64_t ah, uint64_t al, uint64_t bh, uint64_t bl, int E, int neg, int fp32,
                                   uint32_t* out) {
  uint32_t a[5] = {(uint32_t)al, (uint32_t)(al >> 32), (uint32_t)ah, (uint32_t)(ah >> 32), 0u};
  uint32_t b[5] = {(uint32_t)bl, (uint32_t)(bl >> 32), (uint32_t)bh, (uint32_t)(bh >> 32), 0u};
  Rnd r = fp32 ? round_ratio_big<8>(a, b, 5, E, neg, FP32_P, FP32_QMIN, FP32_EMAX)
               : round_ratio_big<8>(a, b, 5, E, neg, BF16_P, BF16_QMIN, BF16_EMAX);
  out[0] = fp32 ? rnd_to_f32_bits(r) : (rnd_to_bf16_bits(r) << 16);
  out[1] = (uint32_t)r.ovf;
}
}  // namespace

extern "C" float ea_round_ratio_cuda(uint64_t a_hi, uint64_t a_lo, uint64_t b_hi, uint64_t b_lo, int E, int neg,
                                     int fp32, int* overflow) {
  uint32_t* d = nullptr;
  uint32_t h[2] = {0, 0};
  if (cudaMalloc(&d, 8) != cudaSuccess) {
    *overflow = -1;
    return 0.0f;
  }
  round_ratio_kernel<<<1, 1>>>(a_hi, a_lo, b_hi, b_lo, E, neg, fp32, d);
  cudaMemcpy(h, d, 8, cudaMemcpyDeviceToHost);
  cudaFree(d);
  *overflow = (int)h[1];
  float f;
  memcpy(&f, &h[0], 4);
  return f;
}

// wide (tier-3) partials of KV shards
extern "C" {

int ea_wide_partials_cuda(const ea_launch_t* a, const int32_t* rows, int n, const ea_wide_partials_t* x,
                          void* stream) {
  int rc = check_launch(a);
  if (rc) return rc;
  if (!x || n < 0 || a->dv > 256 || (n > 0 && !rows)) return -1;
  if (n == 0 || a->rows == 0) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace* w = workspace();
  if (!w) return fail_cuda(cudaGetLastError(), "workspace");
  Prob P;
  build_prob(a, w, P);
  P.export_partials = 1;
  P.w3max = x->maxv;
  P.w3sum = x->sumv;
  P.t3_list = (int*)rows;
  P.t3_fixed = n;
  cudaError_t e = launch_tier3(P, n < 2 * w->sms ? n : 2 * w->sms, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : fail_cuda(e, "wide partials");
}

int ea_wide_partials_rescale_cuda(const ea_wide_partials_t* x, const int64_t* merged_max, int n, int dv,
                                  void* stream) {
  if (!x || !merged_max || n < 0 || dv <= 0 || dv > 256) return -1;
  if (n == 0) return 0;
  Prob P;
  memset(&P, 0, sizeof(P));
  P.dv = dv;
  P.w3max = x->maxv;
  P.w3sum = x->sumv;
  cudaError_t e = launch_wide_rescale(P, n, merged_max, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : fail_cuda(e, "wide rescale");
}

int ea_wide_partials_finalize_cuda(const ea_wide_partials_t* x, const int64_t* merged_max, const int32_t* rows,
                                   int n, int dv, int fp32_out, void* out, uint8_t* flags, int64_t* stats,
                                   void* stream) {
  if (!x || !merged_max || n < 0 || dv <= 0 || dv > 256 || !out || !flags || (n > 0 && !rows)) return -1;
  if (n == 0) return 0;
  Workspace* w;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    w = workspace();
    if (!w) return fail_cuda(cudaGetLastError(), "workspace");
  }
  Prob P;
  memset(&P, 0, sizeof(P));
  P.dv = dv;
  P.fp32 = fp32_out ? 1 : 0;
  P.out = out;
  P.flags = flags;
  P.stats = stats ? (unsigned long long*)stats : w->stats;
  P.w3max = x->maxv;
  P.w3sum = x->sumv;
  P.t3_list = (int*)rows;
  cudaError_t e = launch_wide_finalize(P, n, merged_max, (cudaStream_t)stream);
  return e == cudaSuccess ? 0 : fail_cuda(e, "wide finalize");
}

}  // extern "C"

extern "C" int ea_last_host_stats(int64_t* out) {
  if (!out) return -1;
  memcpy(out, g_last_host_stats, sizeof(g_last_host_stats));
  return 0;
}

extern "C" int ea_set_test_hooks(const ea_test_hooks_t* h) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!h) {
    g_hooks = {0, 0, 0};
    return 0;
  }
  if (h->force_stride < 0 || h->force_tier < 0 || h->force_tier > 2) return -1;
  g_hooks = *h;
  return 0;
}

// Diagnostic: device time of the tier-1 kernel of each ea_launch_cuda call (the hot kernel:
// tensor-core prefill / decode, or the CUDA-core split kernel with its combine).
extern "C" int ea_kernel_timing(int mode, double* total_ms, int64_t* launches) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (mode == 1) {  // on, with a pool of 512 launches
    if (g_kt.ev.empty()) {
      g_kt.ev.resize(1024);
      for (auto& e : g_kt.ev)
        if (cudaEventCreate(&e) != cudaSuccess) return fail_cuda(cudaGetLastError(), "timing events");
    }
    g_kt.used = 0;
    g_kt.on = true;
    return 0;
  }
  if (mode == 2) {  // collect: wait for the recorded launches, sum, reset
    double tot = 0;
    int64_t n = 0;
    for (size_t i = 0; i + 1 < g_kt.used; i += 2) {
      if (cudaEventSynchronize(g_kt.ev[i + 1]) != cudaSuccess) return fail_cuda(cudaGetLastError(), "timing");
      float ms = 0;
      cudaEventElapsedTime(&ms, g_kt.ev[i], g_kt.ev[i + 1]);
      tot += ms;
      ++n;
    }
    if (total_ms) *total_ms = tot;
    if (launches) *launches = n;
    g_kt.used = 0;
    return 0;
  }
  g_kt.on = false;
  return 0;
}

// ---------------------------------------------------------------------------
// host-pointer paged decode (staged copies, synchronous)
// ---------------------------------------------------------------------------
extern "C" int ea_attention_cuda_paged(const uint16_t* q, int64_t batch, int q_heads, int d, const uint16_t* k_cache,
                                       const uint16_t* v_cache, int64_t num_pages, int kv_heads, int page_size, int dv,
                                       float alpha, const int32_t* page_table, int max_pages, const int32_t* seq_lens,
                                       int fp32_out, int splits, void* out, uint8_t* flags, int64_t* stats) {
  if (d <= 0 || d > 1024 || dv <= 0 || splits <= 0 || splits > 65535 || batch < 0 || num_pages < 0 || max_pages <= 0)
    return -1;
  if (q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads != 0 || page_size <= 0) return -9;
  uint32_t ab;
  memcpy(&ab, &alpha, 4);
  int32_t am, ae;
  if (!decode_fp32(ab, am, ae)) return -3;
  const int64_t rows = batch * q_heads;
  if (rows == 0) return 0;
  int64_t maxn = 1;
  for (int64_t b = 0; b < batch; ++b) maxn = std::max<int64_t>(maxn, seq_lens[b]);
  const size_t osz = fp32_out ? 4 : 2;
  const size_t cache = (size_t)num_pages * kv_heads * page_size;
  size_t off = 0;
  auto slot = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~(size_t)255;
    return o;
  };
  size_t oq = slot((size_t)rows * d * 2), ok = slot(cache * d * 2), ov = slot(cache * dv * 2);
  size_t opt = slot((size_t)batch * max_pages * 4), osl = slot((size_t)batch * 4);
  size_t oo = slot((size_t)rows * dv * osz), of = slot((size_t)rows), os = slot(EA_STATS_LEN * 8);
  std::unique_lock<std::mutex> call;
  Workspace* w = host_workspace(off, call);
  if (!w) return -4;
  char* base = (char*)w->stage;
  cudaStream_t st = w->stream;
  cudaError_t e;
  // an error after the first copy waits for the copies in flight before the call returns
  auto fail = [&](cudaError_t err, const char* where) {
    cudaStreamSynchronize(st);
    return fail_cuda(err, where);
  };
  const struct {
    size_t dst;
    const void* src;
    size_t n;
  } h2d[] = {{oq, q, (size_t)rows * d * 2},
             {ok, k_cache, cache * d * 2},
             {ov, v_cache, cache * dv * 2},
             {opt, page_table, (size_t)batch * max_pages * 4},
             {osl, seq_lens, (size_t)batch * 4}};
  for (const auto& c : h2d)
    if (c.n && (e = cudaMemcpyAsync(base + c.dst, c.src, c.n, cudaMemcpyHostToDevice, st)) != cudaSuccess)
      return fail(e, "h2d");
  if ((e = cudaMemsetAsync(base + os, 0, EA_STATS_LEN * 8, st)) != cudaSuccess) return fail(e, "memset");
  ea_launch_t a;
  memset(&a, 0, sizeof(a));
  a.q = (const uint16_t*)(base + oq);
  a.rows = rows;
  a.d = d;
  a.k = (const uint16_t*)(base + ok);
  a.v = (const uint16_t*)(base + ov);
  a.nkeys = (int64_t)cache;
  a.dv = dv;
  a.alpha = alpha;
  a.mask_kind = EA_MASK_PAGED;
  a.page_table = (const int32_t*)(base + opt);
  a.seq_lens = (const int32_t*)(base + osl);
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.max_row_keys = maxn;
  a.fp32_out = fp32_out;
  a.splits = splits;
  a.out = base + oo;
  a.flags = (uint8_t*)(base + of);
  a.stats = (int64_t*)(base + os);
  int rc = launch_host(&a, w);
  if (rc) {
    cudaStreamSynchronize(st);
    return rc;
  }
  int64_t hs[EA_STATS_LEN];
  if ((e = cudaMemcpyAsync(out, base + oo, (size_t)rows * dv * osz, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
      (e = cudaMemcpyAsync(flags, base + of, (size_t)rows, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
      (e = cudaMemcpyAsync(hs, base + os, sizeof(hs), cudaMemcpyDeviceToHost, st)) != cudaSuccess)
    return fail(e, "d2h");
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return fail_cuda(e, "sync");
  if (stats) {
    stats[0] += hs[STAT_SCORE_EXACT];
    stats[1] += hs[STAT_WEIGHT_WIDE];
    stats[2] += hs[STAT_TIER1_UNCERT];
  }
  return wait_status(hs);
}
