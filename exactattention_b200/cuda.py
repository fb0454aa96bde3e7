"""CUDA entry points of certified ExactAttention on B200.

attention_cuda  numpy in / numpy out through the host-pointer C ABI `ea_attention_cuda`: the
                drop-in for the reference's `exactattn.cpu.attention_cpu` (src/exactattn/cpu.py:
                70-109), same signature and return value. Flagged rows are never recomputed on
                the host: every tier runs on the GPU.
launch          torch device tensors in, device tensors out, asynchronous on the current stream,
                through `ea_launch_cuda`: the counterpart of the reference's device-level
                `triton_kernels.launch` (src/exactattn/triton_kernels.py:1324-1351), with CSR,
                per-row key ranges or a paged KV cache as the mask.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from . import _lib
from .formats import ExactAttentionDomainError


@dataclass
class CudaStats:
    """Per-call counters (the reference's CpuStats, cpu.py:54-59, plus the device tiers)."""
    score_fallbacks: int = 0      # scores the window could not certify, recomputed exactly
    weight_fallbacks: int = 0     # weights recomputed by the 128-bit exp2
    final_fallbacks: int = 0      # rows the fast tier left uncertified (rerun by tiers 2 and 3)
    rows: int = 0
    flagged_rows: int = 0         # rows with flag != 0 (domain errors)
    host_fallbacks: int = 0       # always 0


def attention_cuda(q, k, v, alpha, row_ptr=None, key_idx=None, out="bf16", acc_bits=64, tile=64,
                   splits=1, order_seed=0, threads=None, stats: CudaStats | None = None,
                   fallback=True):
    """q: (rows, d) bf16 bits; k: (n, d); v: (n, dv). The mask is CSR (row_ptr, key_idx); None
    means every row attends every key. Returns (out, flags) like attention_cpu; raises
    ExactAttentionDomainError if any row saw a NaN/inf input or an infinite logit.
    `fallback` is accepted for compatibility: nothing is recomputed on the host."""
    lib = _lib.load()
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    rows, d = q.shape
    n, dv = v.shape
    if k.shape[0] != n or k.shape[1] != d:
        raise ValueError("k must be (n, d) with v (n, dv)")
    if row_ptr is not None:
        row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int64)
        key_idx = np.ascontiguousarray(key_idx, dtype=np.int64)
        if row_ptr.shape[0] != rows + 1:
            raise ValueError("row_ptr must have rows + 1 entries")
        if key_idx.size and (key_idx.min() < 0 or key_idx.max() >= n):
            raise ValueError("key_idx out of range")
    fp32 = out == "fp32"
    if out not in ("bf16", "fp32"):
        raise ValueError("out must be 'bf16' or 'fp32'")
    res = np.zeros((rows, dv), dtype=np.float32 if fp32 else np.uint16)
    flags = np.zeros(rows, dtype=np.uint8)
    st = np.zeros(3, dtype=np.int64)
    rc = lib.ea_attention_cuda(q.ctypes.data, rows, d, k.ctypes.data, v.ctypes.data, n, dv,
                               ctypes.c_float(float(np.float32(alpha))),
                               row_ptr.ctypes.data if row_ptr is not None else None,
                               key_idx.ctypes.data if row_ptr is not None else None,
                               int(fp32), acc_bits, tile, splits, order_seed, threads or os.cpu_count() or 1,
                               res.ctypes.data, flags.ctypes.data, st.ctypes.data)
    _lib.check(rc, "ea_attention_cuda")
    if stats is not None:
        stats.score_fallbacks += int(st[0])
        stats.weight_fallbacks += int(st[1])
        stats.final_fallbacks += int(st[2])
        stats.rows += rows
        stats.flagged_rows += int((flags != 0).sum())
    if np.any(flags == 2):
        raise ExactAttentionDomainError("non-finite input or logit overflow")
    if np.any(flags == 1):
        raise RuntimeError("rows left uncertified by every device tier (library bug)")
    return res, flags


def new_stats(device="cuda"):
    """A zeroed device counter array of EA_STATS_LEN int64 (the `stats` argument of launch)."""
    import torch

    return torch.zeros(_lib.EA_STATS_LEN, dtype=torch.int64, device=device)


def round_ratio(a: int, b: int, E: int, neg: bool, fp32: bool) -> tuple[float, bool]:
    """The reference's `cpu.round_ratio` (cpu.py:112-117), evaluated by the device helper."""
    lib = _lib.load()
    ov = ctypes.c_int(0)
    f = lib.ea_round_ratio_cuda(a >> 64, a & ((1 << 64) - 1), b >> 64, b & ((1 << 64) - 1), E, int(neg),
                                int(fp32), ctypes.byref(ov))
    return float(f), bool(ov.value)


# ---------------------------------------------------------------------------
# torch device API
# ---------------------------------------------------------------------------

def _ptr(t):
    return None if t is None else t.data_ptr()


def launch(q, k, v, alpha, *, row_ptr=None, key_idx=None, kv_base=None, kv_len=None, page_table=None,
           seq_lens=None, page_size=0, q_heads=0, kv_heads=0, max_row_keys=None, splits=1, out="bf16",
           out_tensor=None, flags=None, stats=None, stream=None, blocks=None, segments=None, segment_width=0,
           no_alloc=False):
    """Device-level launch, no host sync. q (rows, d), k, v: torch tensors of bf16 bits (any
    16-bit dtype) on one CUDA device. One mask: CSR (row_ptr, key_idx int64), RANGE
    (kv_base, kv_len int64: row r attends k rows kv_base[r] + [0, kv_len[r])), or PAGED
    (page_table (B, max_pages) int32, seq_lens (B,) int32, page_size, q_heads, kv_heads; k/v
    laid out (pages, kv_heads, page_size, d); row r is sequence r // q_heads, head r % q_heads),
    or HYBRID (kv_base/kv_len and row_ptr/key_idx together: the range, then the CSR list).
    max_row_keys bounds every row's key count (required for RANGE/PAGED without a host sync).
    `blocks` (from row_blocks; every row in some block) lets RANGE masks with d = dv = 128 use the
    tensor-core kernel, and HYBRID masks run their shared range on it (the per-row lists on the
    CUDA cores, the two partials merged exactly). `segments` (from row_segments) runs RANGE masks
    with d = dv = 128 through the tensor-core decode kernel (keys on the MMA's M side);
    `segment_width` (optional) is the most rows any segment holds (row_segments' width; a GQA
    group of 2 keeps fewer running sums per thread). PAGED masks with d = dv = 128 and at most 8 q
    heads per kv head take that kernel without a table.
    `no_alloc` calls ea_attention_cuda_noalloc instead: the library allocates no device memory for
    the call (its scratch is a fixed static array of EA_NOALLOC_SCRATCH_BYTES; larger calls raise).
    Returns (out (rows, dv) int16/int32 bit patterns, flags (rows,) uint8)."""
    import torch

    lib = _lib.load()
    dev = q.device
    if dev.type != "cuda":
        raise RuntimeError("launch needs CUDA tensors (there is no CPU path)")
    rows = q.shape[0]
    dv = v.shape[-1]
    if out_tensor is None:
        out_tensor = torch.empty((rows, dv), dtype=torch.int32 if out == "fp32" else torch.int16, device=dev)
    if flags is None:
        flags = torch.empty(rows, dtype=torch.uint8, device=dev)
    a = _launch_args(q, k, v, alpha, row_ptr=row_ptr, key_idx=key_idx, kv_base=kv_base, kv_len=kv_len,
                     page_table=page_table, seq_lens=seq_lens, page_size=page_size, q_heads=q_heads,
                     kv_heads=kv_heads, max_row_keys=max_row_keys, splits=splits, out=out, blocks=blocks,
                     segments=segments, segment_width=segment_width)
    a.out, a.flags = out_tensor.data_ptr(), flags.data_ptr()
    a.stats = _ptr(stats)
    s = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        if no_alloc:
            rc = lib.ea_attention_cuda_noalloc(ctypes.byref(a), ctypes.c_void_p(s))
            if rc != 0:
                msg = lib.ea_noalloc_last_error().decode(errors="replace")
                raise (RuntimeError if rc == -4 else ValueError)(f"{msg} (code {rc})")
        else:
            _lib.check(lib.ea_launch_cuda(ctypes.byref(a), ctypes.c_void_p(s)), "ea_launch_cuda")
    return out_tensor, flags


def _launch_args(q, k, v, alpha, *, row_ptr=None, key_idx=None, kv_base=None, kv_len=None, page_table=None,
                 seq_lens=None, page_size=0, q_heads=0, kv_heads=0, max_row_keys=None, splits=1, out="bf16",
                 blocks=None, segments=None, segment_width=0):
    """ea_launch_t for `launch`'s inputs and mask (outputs left unset)."""
    rows, d = q.shape[0], q.shape[-1]
    dv = v.shape[-1]
    a = _lib.LaunchArgs()
    a.q, a.rows, a.d = q.data_ptr(), rows, d
    a.k, a.v, a.nkeys, a.dv = k.data_ptr(), v.data_ptr(), k.numel() // d, dv
    a.alpha = float(np.float32(alpha))
    if row_ptr is not None and kv_len is not None:
        a.mask_kind = _lib.EA_MASK_HYBRID
        a.row_ptr, a.key_idx = _ptr(row_ptr), _ptr(key_idx)
        a.kv_base, a.kv_len = _ptr(kv_base), _ptr(kv_len)
        if max_row_keys is None:
            max_row_keys = int((kv_len + row_ptr[1:] - row_ptr[:-1]).max().item()) if rows else 1
    elif row_ptr is not None:
        a.mask_kind = _lib.EA_MASK_CSR
        a.row_ptr, a.key_idx = _ptr(row_ptr), _ptr(key_idx)
        if max_row_keys is None:
            max_row_keys = int((row_ptr[1:] - row_ptr[:-1]).max().item()) if rows else 1
    elif kv_len is not None:
        a.mask_kind = _lib.EA_MASK_RANGE
        a.kv_base, a.kv_len = _ptr(kv_base), _ptr(kv_len)
        if max_row_keys is None:
            max_row_keys = int(kv_len.max().item()) if rows else 1
    elif page_table is not None:
        a.mask_kind = _lib.EA_MASK_PAGED
        a.page_table, a.seq_lens = _ptr(page_table), _ptr(seq_lens)
        a.page_size, a.max_pages = int(page_size), int(page_table.shape[-1])
        a.q_heads, a.kv_heads = int(q_heads), int(kv_heads)
        if max_row_keys is None:
            max_row_keys = int(seq_lens.max().item()) if seq_lens.numel() else 1
    else:
        raise ValueError("launch needs a mask: row_ptr/key_idx, kv_base/kv_len or page_table/seq_lens")
    a.max_row_keys = int(max(1, max_row_keys))
    a.fp32_out = int(out == "fp32")
    a.splits = int(splits)
    if blocks is not None:
        a.block_rows, a.nblocks = blocks.data_ptr(), blocks.shape[0]
    if segments is not None:
        a.seg_rows, a.nsegs = segments.data_ptr(), segments.shape[0]
        a.seg_width = int(segment_width)
    return a


class Partials:
    """Row partials of one key range (ea_partials_t) in one flat buffer, the layout of
    EA_PARTIALS_FLAT_BYTES: `i64` (Z, Zerr, N, Nerr) then `i32` (R, status, NR). The flat buffer is
    what one all-gather moves for the merge (ea_partials_merge_gathered_cuda); the two views are
    what the MAX / SUM all-reduce form of the merge reduces."""

    def __init__(self, rows: int, dv: int, device):
        import torch

        self.rows, self.dv = rows, dv
        n64, n32 = rows * (2 + 2 * dv), rows * (2 + dv)
        self.flat = torch.empty(n64 + (n32 + 1) // 2, dtype=torch.int64, device=device)
        self.i64 = self.flat[:n64]
        self.i32 = self.flat[n64:].view(torch.int32)[:n32]
        self._gathered = None
        self.wide_rows = torch.empty(max(1, rows), dtype=torch.int32, device=device)
        self.wide_count = torch.zeros(1, dtype=torch.int32, device=device)
        self.R, self.status = self.i32[:rows], self.i32[rows:2 * rows]
        self.NR = self.i32[2 * rows:].view(rows, dv)
        self.Z, self.Zerr = self.i64[:rows], self.i64[rows:2 * rows]
        self.N = self.i64[2 * rows:(2 + dv) * rows].view(rows, dv)
        self.Nerr = self.i64[(2 + dv) * rows:].view(rows, dv)

    def struct(self) -> "_lib.PartialsArgs":
        p = _lib.PartialsArgs()
        p.R, p.Z, p.Zerr, p.status = (self.R.data_ptr(), self.Z.data_ptr(), self.Zerr.data_ptr(),
                                      self.status.data_ptr())
        p.NR, p.N, p.Nerr = self.NR.data_ptr(), self.N.data_ptr(), self.Nerr.data_ptr()
        return p

    def numpy(self) -> dict:
        return {k: getattr(self, k).cpu().numpy() for k in ("R", "Z", "Zerr", "status", "NR", "N", "Nerr")}

    def gathered(self, world: int):
        """The receive buffer of the all-gather of `world` flat buffers (kept between calls)."""
        import torch

        if self._gathered is None or self._gathered.numel() != world * self.flat.numel():
            self._gathered = torch.empty(world * self.flat.numel(), dtype=torch.int64, device=self.flat.device)
        return self._gathered


def _stream(dev, stream):
    import torch

    return stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream


def partials(q, k, v, alpha, *, parts: Partials | None = None, stream=None, stats=None, **mask) -> Partials:
    """Tier-1 partials of every row over its masked keys (ea_partials_cuda); `mask` takes
    `launch`'s mask keywords (and `splits`, `blocks`). max_row_keys must bound the row's key count
    over ALL key ranges that will be merged, and be the same for each of them."""
    import torch

    lib = _lib.load()
    dev = q.device
    if dev.type != "cuda":
        raise RuntimeError("partials needs CUDA tensors (there is no CPU path)")
    if mask.get("max_row_keys") is None:
        raise ValueError("partials needs max_row_keys (the row's key count over all merged ranges)")
    if parts is None:
        parts = Partials(q.shape[0], v.shape[-1], dev)
    a = _launch_args(q, k, v, alpha, **mask)
    a.stats = _ptr(stats)
    p = parts.struct()
    with torch.cuda.device(dev):
        _lib.check(lib.ea_partials_cuda(ctypes.byref(a), ctypes.byref(p), ctypes.c_void_p(_stream(dev, stream))),
                   "ea_partials_cuda")
    return parts


def rescale_partials(parts: Partials, R_global, NR_global, stream=None) -> None:
    """Re-express `parts` at the merged exponents, in place (ea_partials_rescale_cuda)."""
    import torch

    p = parts.struct()
    dev = parts.i32.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ea_partials_rescale_cuda(ctypes.byref(p), R_global.data_ptr(), NR_global.data_ptr(),
                                                        parts.rows, parts.dv, ctypes.c_void_p(_stream(dev, stream))),
                   "ea_partials_rescale_cuda")


def merge_gathered(gathered, world: int, parts: Partials, max_row_keys: int, out="bf16", stats=None, stream=None):
    """Merge and certified rounding of `world` ranks' gathered flat partials
    (ea_partials_merge_gathered_cuda): (out bits, flags, wide_rows, wide_count) on the device; rows
    flagged 1 are listed in increasing order in wide_rows[:wide_count] (the same list on every
    rank), every later slot -1, for the sharded wide tier."""
    import torch

    dev = parts.flat.device
    o = torch.empty((parts.rows, parts.dv), dtype=torch.int32 if out == "fp32" else torch.int16, device=dev)
    fl = torch.empty(parts.rows, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ea_partials_merge_gathered_cuda(
            gathered.data_ptr(), world, parts.rows, parts.dv, int(max_row_keys), int(out == "fp32"), o.data_ptr(),
            fl.data_ptr(), parts.wide_rows.data_ptr(), parts.wide_count.data_ptr(), _ptr(stats),
            ctypes.c_void_p(_stream(dev, stream))), "ea_partials_merge_gathered_cuda")
    return o, fl, parts.wide_rows, parts.wide_count


def merge_partials_nccl(parts: Partials, nccl_comm: int, stream=None) -> None:
    """The KV-shard merge over a raw NCCL communicator (an ncclComm_t address), in place
    (ea_merge_partials_nccl): the C form of exactattention_b200.dist.merge_partials."""
    import torch

    p = parts.struct()
    dev = parts.i32.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ea_merge_partials_nccl(ctypes.byref(p), parts.rows, parts.dv, ctypes.c_void_p(nccl_comm),
                                                      ctypes.c_void_p(_stream(dev, stream))), "ea_merge_partials_nccl")


def finalize_partials(parts: Partials, max_row_keys: int, out="bf16", stats=None, stream=None):
    """Certified outputs from merged partials (ea_partials_finalize_cuda): (out bits, flags)."""
    import torch

    dev = parts.i32.device
    o = torch.empty((parts.rows, parts.dv), dtype=torch.int32 if out == "fp32" else torch.int16, device=dev)
    fl = torch.empty(parts.rows, dtype=torch.uint8, device=dev)
    p = parts.struct()
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ea_partials_finalize_cuda(ctypes.byref(p), parts.rows, parts.dv, int(max_row_keys),
                                                         int(out == "fp32"), o.data_ptr(), fl.data_ptr(),
                                                         _ptr(stats), ctypes.c_void_p(_stream(dev, stream))),
                   "ea_partials_finalize_cuda")
    return o, fl


def kv_append(k_cache, v_cache, page_table, seq_lens, new_k, new_v, k_meta=None, advance_lens=True,
              stream=None) -> None:
    """Appends new_k / new_v (batch, kv_heads, n_new, d) at positions seq_lens[b] .. of the paged
    caches (pages, kv_heads, page_size, d), through ea_kv_append_cuda; optionally fills k_meta
    (pages, kv_heads, page_size) uint32 (max |k| bits | min nonzero |k| bits << 16) and advances
    seq_lens. All tensors on one CUDA device; no host synchronisation."""
    import torch

    a = _lib.KvAppendArgs()
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.page_table, a.seq_lens = page_table.data_ptr(), seq_lens.data_ptr()
    nk, nv = new_k.contiguous(), new_v.contiguous()  # kept alive until the launch is enqueued
    a.new_k, a.new_v = nk.data_ptr(), nv.data_ptr()
    a.k_meta = _ptr(k_meta)
    a.batch, a.kv_heads, a.n_new, a.d = new_k.shape[0], new_k.shape[1], new_k.shape[2], new_k.shape[3]
    a.page_size, a.max_pages = k_cache.shape[2], page_table.shape[1]
    a.advance_lens = int(advance_lens)
    dev = k_cache.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ea_kv_append_cuda(ctypes.byref(a), ctypes.c_void_p(_stream(dev, stream))),
                   "ea_kv_append_cuda")


def kernel_timing(mode: int) -> tuple[float, int]:
    """ea_kernel_timing: 1 on, 2 collect (summed ms of the tier-1 kernel, launch count), 0 off."""
    ms, n = ctypes.c_double(0), ctypes.c_int64(0)
    _lib.check(_lib.load().ea_kernel_timing(mode, ctypes.byref(ms), ctypes.byref(n)), "ea_kernel_timing")
    return ms.value, n.value


def selftest_fast64(mode: int, seed: int, n: int, stride: int = 1) -> tuple[int, int, int, int]:
    """ea_selftest_fast64: (cases, certified by the binary64 fast path, mismatches, a bad input)."""
    out = (ctypes.c_int64 * 4)()
    _lib.check(_lib.load().ea_selftest_fast64(mode, seed, stride, n, out), "ea_selftest_fast64")
    return tuple(int(x) for x in out)


def reserve_workspace(rows: int, splits: int, dv: int) -> None:
    _lib.check(_lib.load().ea_reserve_workspace(rows, splits, dv), "ea_reserve_workspace")


def release() -> None:
    _lib.load().ea_cuda_release()


def attention_cuda_ranges(q, k, v, alpha, kv_base, kv_len, max_row_keys=None, out="bf16", splits=1,
                          stats: CudaStats | None = None, out_buf=None, flags_buf=None):
    """Host buffers through `ea_attention_cuda_ranges`: row r attends k rows
    kv_base[r] + [0, kv_len[r]). Host arrays may be pinned (torch pin_memory) numpy views.
    Returns (out, flags); raises like attention_cuda."""
    lib = _lib.load()
    rows, d = q.shape
    n, dv = v.shape
    fp32 = out == "fp32"
    res = out_buf if out_buf is not None else np.zeros((rows, dv), dtype=np.float32 if fp32 else np.uint16)
    flags = flags_buf if flags_buf is not None else np.zeros(rows, dtype=np.uint8)
    st = np.zeros(3, dtype=np.int64)
    mk = int(max_row_keys if max_row_keys is not None else (kv_len.max() if rows else 1))
    rc = lib.ea_attention_cuda_ranges(q.ctypes.data, rows, d, k.ctypes.data, v.ctypes.data, n, dv,
                                      ctypes.c_float(float(np.float32(alpha))), kv_base.ctypes.data,
                                      kv_len.ctypes.data, mk, int(fp32), splits, res.ctypes.data, flags.ctypes.data,
                                      st.ctypes.data)
    _lib.check(rc, "ea_attention_cuda_ranges")
    if stats is not None:
        stats.score_fallbacks += int(st[0])
        stats.weight_fallbacks += int(st[1])
        stats.final_fallbacks += int(st[2])
        stats.rows += rows
        stats.flagged_rows += int((flags != 0).sum())
    if np.any(flags == 2):
        raise ExactAttentionDomainError("non-finite input or logit overflow")
    if np.any(flags == 1):
        raise RuntimeError("rows left uncertified by every device tier (library bug)")
    return res, flags


def attention_cuda_paged(q, k_cache, v_cache, alpha, page_table, seq_lens, q_heads: int, out="bf16", splits=1,
                         stats: CudaStats | None = None, out_buf=None, flags_buf=None):
    """Host buffers through `ea_attention_cuda_paged`: q (batch * q_heads, d), caches
    (num_pages, kv_heads, page_size, d), page_table (batch, max_pages) int32, seq_lens (batch,)
    int32. Returns (out, flags); raises like attention_cuda."""
    lib = _lib.load()
    rows, d = q.shape
    npg, hkv, ps, dv = v_cache.shape
    batch = rows // q_heads
    fp32 = out == "fp32"
    res = out_buf if out_buf is not None else np.zeros((rows, dv), dtype=np.float32 if fp32 else np.uint16)
    flags = flags_buf if flags_buf is not None else np.zeros(rows, dtype=np.uint8)
    st = np.zeros(3, dtype=np.int64)
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    rc = lib.ea_attention_cuda_paged(q.ctypes.data, batch, q_heads, d, k_cache.ctypes.data, v_cache.ctypes.data, npg,
                                     hkv, ps, dv, ctypes.c_float(float(np.float32(alpha))), pt.ctypes.data,
                                     pt.shape[1], sl.ctypes.data, int(fp32), splits, res.ctypes.data,
                                     flags.ctypes.data, st.ctypes.data)
    _lib.check(rc, "ea_attention_cuda_paged")
    if stats is not None:
        stats.score_fallbacks += int(st[0])
        stats.weight_fallbacks += int(st[1])
        stats.final_fallbacks += int(st[2])
        stats.rows += rows
        stats.flagged_rows += int((flags != 0).sum())
    if np.any(flags == 2):
        raise ExactAttentionDomainError("non-finite input or logit overflow")
    if np.any(flags == 1):
        raise RuntimeError("rows left uncertified by every device tier (library bug)")
    return res, flags


def split_runs(row_ptr: np.ndarray, key_idx: np.ndarray):
    """CSR rows of ascending, distinct keys (the rows of a boolean mask) as a leading run of
    consecutive keys plus a tail list: (kv_base, kv_len, tail_row_ptr, tail_key_idx). Causal and
    prefix rows are one run with an empty tail; tree rows are the prefix run plus the ancestors.
    The same keys in either layout give the same bits."""
    row_ptr = np.asarray(row_ptr, np.int64)
    key_idx = np.asarray(key_idx, np.int64)
    rows = len(row_ptr) - 1
    counts = np.diff(row_ptr)
    kb = np.zeros(rows, np.int64)
    nz = counts > 0
    kb[nz] = key_idx[row_ptr[:-1][nz]]
    rowid = np.repeat(np.arange(rows), counts)
    offs = np.arange(len(key_idx), dtype=np.int64) - np.repeat(row_ptr[:-1], counts)
    # keys ascending and distinct: key - (first + offset) never decreases along a row, so the
    # positions still in the run are a prefix of the row
    inrun = key_idx == kb[rowid] + offs
    kl = np.bincount(rowid[inrun], minlength=rows).astype(np.int64)
    tail = key_idx[~inrun]
    trp = np.concatenate([[0], np.cumsum(counts - kl)]).astype(np.int64)
    return kb, kl, trp, tail


def mask_launch_kwargs(row_ptr: np.ndarray, key_idx: np.ndarray, d: int, dv: int, device):
    """`launch` mask keywords for a CSR mask of ascending, distinct keys: RANGE when every row is
    one run of consecutive keys, HYBRID when runs hold at least three quarters of the keys (at
    d = dv = 128), CSR otherwise; with the row blocks or decode segments that put RANGE and HYBRID
    masks on the tensor-core kernels."""
    import torch

    kb, kl, trp, tail = split_runs(row_ptr, key_idx)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(device)  # noqa: E731
    counts = np.diff(np.asarray(row_ptr, np.int64))
    mk = int(counts.max(initial=1))
    tc = d == 128 and dv == 128
    if len(tail) == 0:
        kw = dict(kv_base=t(kb), kv_len=t(kl), max_row_keys=mk)
        if tc:
            groups = np.unique(kb, return_counts=True)[1]
            if len(groups) and groups.max() <= 8:
                kw["segments"] = t(row_segments(kb))
                kw["segment_width"] = int(groups.max())
            else:
                kw["blocks"] = t(row_blocks(kb, kl))
        return kw
    if tc and 4 * len(tail) <= len(key_idx):
        return dict(kv_base=t(kb), kv_len=t(kl), row_ptr=t(trp), key_idx=t(tail), max_row_keys=mk,
                    blocks=t(row_blocks(kb, kl)))
    return dict(row_ptr=t(np.asarray(row_ptr, np.int64)), key_idx=t(np.asarray(key_idx, np.int64)), max_row_keys=mk)


def row_segments(kv_base: np.ndarray, width: int = 8) -> np.ndarray:
    """Groups RANGE-mask rows that share kv_base into segments of at most `width` (8) rows, -1
    padded: the (nsegs, 8) int32 `segments` argument of launch (decode: a GQA group per segment).
    Any grouping gives the same bits."""
    kv_base = np.asarray(kv_base, np.int64)
    order = np.argsort(kv_base, kind="stable")
    b = kv_base[order]
    cuts = np.flatnonzero(np.diff(b)) + 1
    out = []
    for grp in np.split(order, cuts):
        for c in range(0, len(grp), width):
            seg = np.full(8, -1, np.int32)
            part = grp[c:c + width]
            seg[:len(part)] = part
            out.append(seg)
    return np.stack(out) if out else np.zeros((0, 8), np.int32)


def row_blocks(kv_base: np.ndarray, kv_len: np.ndarray, bm: int = 128) -> np.ndarray:
    """Groups RANGE-mask rows that share kv_base into blocks of `bm` (longest rows first, blocks
    ordered longest first, -1 padding): the (nblocks, bm) int32 `blocks` argument of launch. The
    grouping is a schedule only: any grouping gives the same bits."""
    kv_base = np.asarray(kv_base, np.int64)
    kv_len = np.asarray(kv_len, np.int64)
    order = np.lexsort((-kv_len, kv_base))
    b = kv_base[order]
    cuts = np.flatnonzero(np.diff(b)) + 1
    out = []
    for grp in np.split(order, cuts):
        for c in range(0, len(grp), bm):
            blk = np.full(bm, -1, np.int32)
            part = grp[c:c + bm]
            blk[:len(part)] = part
            out.append(blk)
    if not out:
        return np.zeros((0, bm), np.int32)
    arr = np.stack(out)
    first_len = kv_len[arr[:, 0]]
    return arr[np.argsort(-first_len, kind="stable")]


class WidePartials:
    """Wide (tier-3) partials of `n` listed rows (ea_wide_partials_t): `maxv` (n, 4) int64 merged
    by MAX, `sumv` (n, dv + 1, WIDE_DIGITS + 1) int64 merged by SUM."""

    def __init__(self, n: int, dv: int, device):
        import torch

        self.n, self.dv = n, dv
        self.maxv = torch.empty((n, 4), dtype=torch.int64, device=device)
        self.sumv = torch.empty((n, dv + 1, _lib.WIDE_DIGITS + 1), dtype=torch.int64, device=device)

    def struct(self) -> "_lib.WidePartialsArgs":
        w = _lib.WidePartialsArgs()
        w.maxv, w.sumv = self.maxv.data_ptr(), self.sumv.data_ptr()
        return w


def wide_partials(q, k, v, alpha, rows, *, stream=None, stats=None, **mask) -> WidePartials:
    """Wide partials over this key range of the rows listed in `rows` (int32 device tensor),
    ea_wide_partials_cuda; `mask` as for `partials` (max_row_keys required)."""
    import torch

    lib = _lib.load()
    dev = q.device
    if mask.get("max_row_keys") is None:
        raise ValueError("wide_partials needs max_row_keys (the row's key count over all merged ranges)")
    rows = rows.to(device=dev, dtype=torch.int32).contiguous()
    w = WidePartials(rows.numel(), v.shape[-1], dev)
    mask = {k_: v_ for k_, v_ in mask.items() if k_ not in ("blocks", "segments", "segment_width", "splits")}
    a = _launch_args(q, k, v, alpha, **mask)
    a.stats = _ptr(stats)
    ws = w.struct()
    with torch.cuda.device(dev):
        _lib.check(lib.ea_wide_partials_cuda(ctypes.byref(a), rows.data_ptr(), w.n, ctypes.byref(ws),
                                             ctypes.c_void_p(_stream(dev, stream))), "ea_wide_partials_cuda")
    return w


def rescale_wide_partials(w: WidePartials, merged_max, stream=None) -> None:
    import torch

    ws = w.struct()
    dev = w.maxv.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ea_wide_partials_rescale_cuda(ctypes.byref(ws), merged_max.data_ptr(), w.n, w.dv,
                                                             ctypes.c_void_p(_stream(dev, stream))),
                   "ea_wide_partials_rescale_cuda")


def finalize_wide_partials(w: WidePartials, merged_max, rows, out_tensor, flags, out="bf16", stats=None,
                           stream=None) -> None:
    """Writes the listed rows of out_tensor / flags from merged wide partials."""
    import torch

    ws = w.struct()
    dev = w.maxv.device
    rows = rows.to(device=dev, dtype=torch.int32).contiguous()
    with torch.cuda.device(dev):
        _lib.check(_lib.load().ea_wide_partials_finalize_cuda(ctypes.byref(ws), merged_max.data_ptr(), rows.data_ptr(),
                                                              w.n, w.dv, int(out == "fp32"), out_tensor.data_ptr(),
                                                              flags.data_ptr(), _ptr(stats),
                                                              ctypes.c_void_p(_stream(dev, stream))),
                   "ea_wide_partials_finalize_cuda")
