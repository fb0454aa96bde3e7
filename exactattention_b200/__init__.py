"""Certified ExactAttention on B200 (sm_100a): the reference's Python API, computed by
hand-written CUDA through a C-ABI library (libexactattn_cuda.so).

Same names and semantics as the reference package `exactattn` (src/exactattn/__init__.py:3-14):
`attention(q_bits, k_bits, v_bits, alpha, mask=None, out="bf16")` returns the spec's bits for
every row, or raises ExactAttentionDomainError. There is no CPU path: without the library or a
GPU these calls raise.
"""

from __future__ import annotations

import numpy as np

from .formats import ExactAttentionDomainError, bf16_bits_to_float32, default_alpha, float_to_bf16_bits

__all__ = [
    "ExactAttentionDomainError",
    "attention",
    "attention_row",
    "bf16_bits_to_float32",
    "default_alpha",
    "float_to_bf16_bits",
]


def _csr_from_mask(mask: np.ndarray):
    mask = np.asarray(mask, dtype=bool)
    row_ptr = np.concatenate([[0], np.cumsum(mask.sum(axis=1))]).astype(np.int64)
    key_idx = (np.concatenate([np.flatnonzero(m) for m in mask]).astype(np.int64)
               if mask.size else np.zeros(0, np.int64))
    return row_ptr, key_idx


def attention(q_bits, k_bits, v_bits, alpha, mask=None, out: str = "bf16") -> np.ndarray:
    """q (r, d), k (n, d), v (n, dv) bf16 bit patterns; mask (r, n) bool or None.
    The reference's `exactattn.attention` (reference.py:150-161), computed on the GPU."""
    from .cuda import attention_cuda

    q_bits = np.asarray(q_bits, dtype=np.uint16)
    k_bits = np.asarray(k_bits, dtype=np.uint16)
    v_bits = np.asarray(v_bits, dtype=np.uint16)
    if mask is None:
        row_ptr = key_idx = None
    else:
        row_ptr, key_idx = _csr_from_mask(mask)
    res, _ = attention_cuda(q_bits, k_bits, v_bits, alpha, row_ptr, key_idx, out=out)
    return res


def attention_row(q_bits, k_bits, v_bits, alpha, out: str = "bf16") -> np.ndarray:
    """One query row against every given key (reference.py:146)."""
    q = np.asarray(q_bits, dtype=np.uint16).reshape(1, -1)
    k = np.asarray(k_bits, dtype=np.uint16).reshape(-1, q.shape[1])
    v = np.asarray(v_bits, dtype=np.uint16)
    v = v.reshape(k.shape[0], -1) if v.size else v.reshape(0, v.shape[-1] if v.ndim == 2 else 0)
    return attention(q, k, v, alpha, None, out)[0]
