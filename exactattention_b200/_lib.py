"""Loads libexactattn_cuda.so (built in-tree by build.py) and declares its C ABI
(include/exactattn_cuda.h). There is no CPU fallback: a missing library or a missing GPU raises."""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libexactattn_cuda.so")
_lib = None

EA_MASK_CSR, EA_MASK_RANGE, EA_MASK_PAGED, EA_MASK_HYBRID = 0, 1, 2, 3
EA_STATS_LEN = 12
STAT_NAMES = ("score_exact", "weight_wide", "tier1_uncertified", "domain_rows", "unresolved_rows", "pairs",
              "host_fallbacks", "tc_pairs", "waits_expired", "tier2_uncertified", "tier2_pairs", "forced_rows")
# return codes (include/exactattn_cuda.h)
RC_WAIT_EXPIRED = -5

# Every symbol include/exactattn_cuda.h declares.
EXPORTS = ("ea_attention_cuda", "ea_attention_cuda_ranges", "ea_round_ratio_cuda", "ea_launch_cuda",
           "ea_reserve_workspace", "ea_cuda_release", "ea_cuda_last_error", "ea_attention_cuda_noalloc",
           "ea_noalloc_last_error", "ea_partials_cuda", "ea_partials_rescale_cuda", "ea_partials_finalize_cuda",
           "ea_wide_partials_cuda", "ea_wide_partials_rescale_cuda", "ea_wide_partials_finalize_cuda",
           "ea_kernel_timing", "ea_attention_cuda_paged", "ea_kv_append_cuda", "ea_selftest_fast64",
           "ea_merge_partials_nccl", "ea_set_test_hooks", "ea_last_host_stats",
           "ea_partials_merge_gathered_cuda")
WIDE_DIGITS = 48  # EA_WIDE_DIGITS


class LaunchArgs(ctypes.Structure):
    """ea_launch_t (include/exactattn_cuda.h), field for field."""
    _fields_ = [
        ("q", ctypes.c_void_p), ("rows", ctypes.c_int64), ("d", ctypes.c_int),
        ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("nkeys", ctypes.c_int64), ("dv", ctypes.c_int),
        ("alpha", ctypes.c_float),
        ("mask_kind", ctypes.c_int),
        ("row_ptr", ctypes.c_void_p), ("key_idx", ctypes.c_void_p),
        ("kv_base", ctypes.c_void_p), ("kv_len", ctypes.c_void_p),
        ("page_table", ctypes.c_void_p), ("seq_lens", ctypes.c_void_p),
        ("page_size", ctypes.c_int), ("max_pages", ctypes.c_int), ("q_heads", ctypes.c_int),
        ("kv_heads", ctypes.c_int),
        ("max_row_keys", ctypes.c_int64),
        ("fp32_out", ctypes.c_int), ("splits", ctypes.c_int),
        ("out", ctypes.c_void_p), ("flags", ctypes.c_void_p), ("stats", ctypes.c_void_p),
        ("block_rows", ctypes.c_void_p), ("nblocks", ctypes.c_int64),
        ("seg_rows", ctypes.c_void_p), ("nsegs", ctypes.c_int64), ("seg_width", ctypes.c_int),
    ]


class PartialsArgs(ctypes.Structure):
    """ea_partials_t (include/exactattn_cuda.h)."""
    _fields_ = [("R", ctypes.c_void_p), ("Z", ctypes.c_void_p), ("Zerr", ctypes.c_void_p),
                ("status", ctypes.c_void_p), ("NR", ctypes.c_void_p), ("N", ctypes.c_void_p),
                ("Nerr", ctypes.c_void_p)]


class WidePartialsArgs(ctypes.Structure):
    """ea_wide_partials_t (include/exactattn_cuda.h)."""
    _fields_ = [("maxv", ctypes.c_void_p), ("sumv", ctypes.c_void_p)]


class TestHooks(ctypes.Structure):
    """ea_test_hooks_t (include/exactattn_cuda.h)."""
    _fields_ = [("force_stride", ctypes.c_int), ("force_tier", ctypes.c_int), ("wait_debug", ctypes.c_int)]


class KvAppendArgs(ctypes.Structure):
    """ea_kv_append_t (include/exactattn_cuda.h)."""
    _fields_ = [("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p), ("page_table", ctypes.c_void_p),
                ("seq_lens", ctypes.c_void_p), ("new_k", ctypes.c_void_p), ("new_v", ctypes.c_void_p),
                ("k_meta", ctypes.c_void_p), ("batch", ctypes.c_int64), ("kv_heads", ctypes.c_int),
                ("page_size", ctypes.c_int), ("max_pages", ctypes.c_int), ("n_new", ctypes.c_int),
                ("d", ctypes.c_int), ("advance_lens", ctypes.c_int)]


def load(path: str | None = None):
    """The library handle, with argument types declared. Raises if it is not built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"{p} is missing: build it with `python -m exactattention_b200.build`")
    lib = ctypes.CDLL(p)
    P = ctypes.c_void_p
    lib.ea_attention_cuda.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_float, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_uint64, ctypes.c_int, P, P, P]
    lib.ea_attention_cuda.restype = ctypes.c_int
    lib.ea_attention_cuda_ranges.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int64, ctypes.c_int,
                                             ctypes.c_float, P, P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P, P,
                                             P]
    lib.ea_attention_cuda_ranges.restype = ctypes.c_int
    lib.ea_round_ratio_cuda.argtypes = [ctypes.c_uint64] * 4 + [ctypes.c_int] * 3 + [ctypes.POINTER(ctypes.c_int)]
    lib.ea_round_ratio_cuda.restype = ctypes.c_float
    lib.ea_launch_cuda.argtypes = [ctypes.POINTER(LaunchArgs), P]
    lib.ea_launch_cuda.restype = ctypes.c_int
    lib.ea_attention_cuda_noalloc.argtypes = [ctypes.POINTER(LaunchArgs), P]
    lib.ea_attention_cuda_noalloc.restype = ctypes.c_int
    lib.ea_noalloc_last_error.argtypes = []
    lib.ea_noalloc_last_error.restype = ctypes.c_char_p
    lib.ea_partials_cuda.argtypes = [ctypes.POINTER(LaunchArgs), ctypes.POINTER(PartialsArgs), P]
    lib.ea_partials_cuda.restype = ctypes.c_int
    lib.ea_partials_rescale_cuda.argtypes = [ctypes.POINTER(PartialsArgs), P, P, ctypes.c_int64, ctypes.c_int, P]
    lib.ea_partials_rescale_cuda.restype = ctypes.c_int
    lib.ea_partials_finalize_cuda.argtypes = [ctypes.POINTER(PartialsArgs), ctypes.c_int64, ctypes.c_int,
                                              ctypes.c_int64, ctypes.c_int, P, P, P, P]
    lib.ea_partials_finalize_cuda.restype = ctypes.c_int
    W = ctypes.POINTER(WidePartialsArgs)
    lib.ea_wide_partials_cuda.argtypes = [ctypes.POINTER(LaunchArgs), P, ctypes.c_int, W, P]
    lib.ea_wide_partials_cuda.restype = ctypes.c_int
    lib.ea_wide_partials_rescale_cuda.argtypes = [W, P, ctypes.c_int, ctypes.c_int, P]
    lib.ea_wide_partials_rescale_cuda.restype = ctypes.c_int
    lib.ea_wide_partials_finalize_cuda.argtypes = [W, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, P]
    lib.ea_wide_partials_finalize_cuda.restype = ctypes.c_int
    lib.ea_attention_cuda_paged.argtypes = [P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int64,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, P, ctypes.c_int,
                                            P, ctypes.c_int, ctypes.c_int, P, P, P]
    lib.ea_attention_cuda_paged.restype = ctypes.c_int
    lib.ea_kv_append_cuda.argtypes = [ctypes.POINTER(KvAppendArgs), P]
    lib.ea_kv_append_cuda.restype = ctypes.c_int
    lib.ea_kernel_timing.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]
    lib.ea_kernel_timing.restype = ctypes.c_int
    lib.ea_selftest_fast64.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int64, P]
    lib.ea_selftest_fast64.restype = ctypes.c_int
    lib.ea_merge_partials_nccl.argtypes = [ctypes.POINTER(PartialsArgs), ctypes.c_int64, ctypes.c_int, P, P]
    lib.ea_merge_partials_nccl.restype = ctypes.c_int
    lib.ea_partials_merge_gathered_cuda.argtypes = [P, ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int64,
                                                    ctypes.c_int, P, P, P, P, P, P]
    lib.ea_partials_merge_gathered_cuda.restype = ctypes.c_int
    lib.ea_last_host_stats.argtypes = [P]
    lib.ea_last_host_stats.restype = ctypes.c_int
    lib.ea_set_test_hooks.argtypes = [ctypes.POINTER(TestHooks)]
    lib.ea_set_test_hooks.restype = ctypes.c_int
    lib.ea_reserve_workspace.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int]
    lib.ea_reserve_workspace.restype = ctypes.c_int
    lib.ea_cuda_release.argtypes = []
    lib.ea_cuda_release.restype = None
    lib.ea_cuda_last_error.argtypes = []
    lib.ea_cuda_last_error.restype = ctypes.c_char_p
    if path is None:
        _lib = lib
    return lib


class WaitExpiredWarning(RuntimeWarning):
    """A bounded device wait gave up during a synchronous call (code -5): the GPU stalled. The
    affected rows were recomputed by the later tiers, so the call's outputs are exact."""


def check(rc: int, what: str) -> None:
    if rc == 0:
        return
    lib = load()
    msg = lib.ea_cuda_last_error().decode(errors="replace")
    if rc == -1:
        raise ValueError(f"{what}: invalid dimensions (code -1)")
    if rc == -2:
        raise ValueError(f"{what}: acc_bits must be 64 or 128 (code -2)")
    if rc == -3:
        raise ValueError(f"{what}: alpha is not finite (code -3)")
    if rc == RC_WAIT_EXPIRED:
        import warnings

        warnings.warn(f"{what}: {msg} (code -5)", WaitExpiredWarning, stacklevel=3)
        return
    if rc == -9:
        raise ValueError(f"{what}: unsupported layout (code -9)")
    raise RuntimeError(f"{what}: CUDA error (code {rc}): {msg}")


def set_test_hooks(force_stride: int = 0, force_tier: int = 0, wait_debug: int = 0) -> None:
    """ea_set_test_hooks (tests only): force rows out of tier 1 (and tier 2), or make the bounded
    waits of the tensor-core kernels report expiry. All zero restores production behaviour."""
    h = TestHooks(force_stride, force_tier, wait_debug)
    rc = load().ea_set_test_hooks(ctypes.byref(h))
    if rc:
        raise ValueError("invalid test hooks")


def last_host_stats() -> dict:
    """The full counters of this thread's last host-pointer call (ea_last_host_stats)."""
    import numpy as np

    out = np.zeros(EA_STATS_LEN, np.int64)
    load().ea_last_host_stats(out.ctypes.data)
    return dict(zip(STAT_NAMES, (int(x) for x in out)))
