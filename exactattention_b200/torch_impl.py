"""`attention_torch`: the reference's torch entry point (src/exactattn/torch_impl.py:178-335), same
signature and return value, served by the CUDA kernels. `device` must be a CUDA device: the
reference ran it as int64 tensor ops on any device; here the B200 kernels do the work."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class TorchStats:
    rows: int = 0
    flagged_rows: int = 0
    oracle_weights: int = 0   # always 0: weights never leave the device


def attention_torch(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, alpha, mask: np.ndarray,
                    device: str = "cuda", out: str = "bf16", tile: int = 64, row_chunk: int = 64,
                    tile_order_seed: int | None = None, stats: TorchStats | None = None,
                    fallback: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """q: (R, d), k: (n, d), v: (n, dv) bf16 bits; mask: (R, n) bool. Returns (out, flags) with
    flags 0 (certified on the device) or 2 (domain error). tile, row_chunk, tile_order_seed and
    fallback are accepted for compatibility; they cannot change the bits."""
    import torch

    from . import cuda

    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("attention_torch runs on the CUDA kernels: pass a cuda device")
    q = np.ascontiguousarray(q_bits, dtype=np.uint16)
    k = np.ascontiguousarray(k_bits, dtype=np.uint16)
    v = np.ascontiguousarray(v_bits, dtype=np.uint16)
    mask = np.asarray(mask, dtype=bool)
    counts = mask.sum(axis=1)
    row_ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    key_idx = np.concatenate([np.flatnonzero(m) for m in mask]).astype(np.int64) if mask.size else np.zeros(0, np.int64)

    def t(x, dt):
        return torch.from_numpy(x.view(dt) if x.dtype == np.uint16 else x).to(dev)

    Q, K, V = t(q, np.int16), t(k, np.int16), t(v, np.int16)
    # causal / prefix rows as key ranges, tree rows as a range plus a list: the tensor-core kernels
    mask_kw = cuda.mask_launch_kwargs(row_ptr, key_idx, q.shape[1], v.shape[1], dev)
    o, fl = cuda.launch(Q, K, V, alpha, out=out, **mask_kw)
    o = o.cpu().numpy()
    flags = fl.cpu().numpy().astype(np.uint8)
    res = o.view(np.float32).copy() if out == "fp32" else o.view(np.uint16).copy()
    if np.any(flags == 1):
        raise RuntimeError("rows left uncertified by every device tier (library bug)")
    if stats is not None:
        stats.rows += q.shape[0]
        stats.flagged_rows += int((flags != 0).sum())
    return res, flags
