"""ctypes driver for the reference's own certified C++ kernel, built into oracle/_ref/.

TEST INFRASTRUCTURE ONLY (tests/, __graft_entry__.smoke(), bench.py's CPU-baseline leg).

`attention_ref` mirrors the reference's `cpu.attention_cpu` (src/exactattn/cpu.py:70-109):
the C++ kernel certifies what it can (flags 0), rows it flags 1 are recomputed by the exact
oracle (oracle/exact.py), and a flag 2 (non-finite input) raises. The library's entry point
`ea_attention_cpu` is declared at csrc/exact_attention_cpu.cpp:585-588 of the reference.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from . import exact

_HERE = os.path.dirname(os.path.abspath(__file__))
_VARIANTS = (("x86-64-v4", "libexactattn_cpu_v4.so", {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"}),
             ("x86-64-v3", "libexactattn_cpu_v3.so", {"avx2", "bmi2", "fma", "movbe"}),
             ("x86-64-v2", "libexactattn_cpu.so", set()))
_lib = None


def _cpu_flags() -> set:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("flags"):
                return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def _pick() -> tuple[str, str]:
    """The most capable build of the reference kernel this CPU runs (the reference builds with
    -march=native; oracle/Makefile builds the x86-64 levels)."""
    flags = _cpu_flags()
    for name, so, need in _VARIANTS:
        p = os.path.join(_HERE, "_ref", so)
        if os.path.exists(p) and need <= flags:
            return name, p
    return _VARIANTS[-1][0], os.path.join(_HERE, "_ref", _VARIANTS[-1][1])


LIB_VARIANT, LIB_PATH = _pick()


def available() -> bool:
    return os.path.exists(LIB_PATH)


def build_variant() -> str:
    return LIB_VARIANT


def _load():
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{LIB_PATH} is not built (make -C oracle)")
        lib = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        lib.ea_attention_cpu.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int64, ctypes.c_int,
                                         ctypes.c_float, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_uint64, ctypes.c_int, P, P, P]
        lib.ea_attention_cpu.restype = ctypes.c_int
        lib.ea_round_ratio.argtypes = [ctypes.c_uint64] * 4 + [ctypes.c_int] * 3 + [ctypes.POINTER(ctypes.c_int)]
        lib.ea_round_ratio.restype = ctypes.c_float
        _lib = lib
    return _lib


@dataclass
class RefStats:
    score_fallbacks: int = 0
    weight_fallbacks: int = 0
    final_fallbacks: int = 0
    rows: int = 0
    flagged_rows: int = 0


def attention_ref(q, k, v, alpha, row_ptr=None, key_idx=None, out="bf16", acc_bits=64, tile=64,
                  splits=1, order_seed=0, threads=None, stats: RefStats | None = None,
                  fallback=True):
    """(out, flags) exactly as the reference's attention_cpu returns them."""
    lib = _load()
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    rows, d = q.shape
    n, dv = v.shape
    if row_ptr is None:
        row_ptr = np.arange(rows + 1, dtype=np.int64) * n
        key_idx = np.tile(np.arange(n, dtype=np.int64), rows)
    row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int64)
    key_idx = np.ascontiguousarray(key_idx, dtype=np.int64)
    fp32 = out == "fp32"
    res = np.zeros((rows, dv), dtype=np.float32 if fp32 else np.uint16)
    flags = np.zeros(rows, dtype=np.uint8)
    st = np.zeros(3, dtype=np.int64)
    threads = threads or os.cpu_count() or 1
    rc = lib.ea_attention_cpu(q.ctypes.data, rows, d, k.ctypes.data, v.ctypes.data, n, dv,
                              ctypes.c_float(float(np.float32(alpha))), row_ptr.ctypes.data,
                              key_idx.ctypes.data, int(fp32), acc_bits, tile, splits, order_seed,
                              threads, res.ctypes.data, flags.ctypes.data, st.ctypes.data)
    if rc != 0:
        raise ValueError(f"ea_attention_cpu: invalid arguments (code {rc})")
    if stats is not None:
        stats.score_fallbacks += int(st[0])
        stats.weight_fallbacks += int(st[1])
        stats.final_fallbacks += int(st[2])
        stats.rows += rows
        stats.flagged_rows += int((flags != 0).sum())
    if np.any(flags == 2):
        raise exact.ExactAttentionDomainError("non-finite input")
    if fallback:
        for r in np.flatnonzero(flags):
            sel = key_idx[row_ptr[r]:row_ptr[r + 1]]
            res[r] = exact.attention_row(q[r], k[sel], v[sel], alpha, out)
    return res, flags


def round_ratio(a: int, b: int, E: int, neg: bool, fp32: bool) -> tuple[float, bool]:
    """The reference's exported ea_round_ratio (cpp:632-638)."""
    lib = _load()
    ov = ctypes.c_int(0)
    f = lib.ea_round_ratio(a >> 64, a & ((1 << 64) - 1), b >> 64, b & ((1 << 64) - 1), E, int(neg), int(fp32),
                           ctypes.byref(ov))
    return float(f), bool(ov.value)
