"""Long rows sharded by key range over ranks (one process per GPU), merged exactly.

Each rank holds a contiguous key range of every (sequence, kv head) and computes the row
partials of its range (`cuda.partials`): a reference exponent R and the fixed-point sums Z, N
with their error bounds. The merge is the split-KV combine of the reference's certified kernel
(triton_kernels.py:1081 `_ea_combine_kernel`; certified.py:213-246 `merge`), spread over ranks:

  1. all-reduce MAX of (R, status, NR)            one int32 message of rows x (2 + dv)
  2. every rank re-expresses its sums at the maxima (floor shifts; the error grows by one unit
     per shifted value), so all ranks' integers are in the same units
  3. all-reduce SUM of (Z, Zerr, N, Nerr)         one int64 message of rows x (2 + 2 dv)
  4. certified rounding of the merged interval on every rank.

Rows whose merged interval does not certify (flag 1; the same rows on every rank, since every
rank rounds the same merged integers) take the wide tier the same way: each rank accumulates its
keys of those rows into 1536-bit windows (`cuda.wide_partials`), MAX all-reduce of the reference
exponents, shift to the maximum, SUM all-reduce of the 32-bit digits, certified rounding.

MAX and SUM are associative and commutative on integers, so the result is the same for every
rank count, rank order and reduction tree: the bits do not depend on how the keys were sharded.
The fixed-point headroom comes from the row's key count over ALL ranks (max_row_keys), so the
int64 SUMs cannot overflow.
"""

from __future__ import annotations

from . import cuda


def merge_partials(parts: "cuda.Partials", group=None, rescale=None) -> "cuda.Partials":
    """Steps 1-3 in place on `parts`. `rescale(parts, R_global, NR_global)` defaults to the
    device kernel; every rank must call this with the same row count and dv."""
    import torch.distributed as dist

    rows = parts.rows
    mx = parts.i32.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    (rescale or cuda.rescale_partials)(parts, mx[:rows], mx[2 * rows:].view(rows, parts.dv))
    parts.status.copy_(mx[rows:2 * rows])
    dist.all_reduce(parts.i64, op=dist.ReduceOp.SUM, group=group)
    return parts


def wide_tier(q, k, v, alpha, rows, out_tensor, flags, *, max_row_keys: int, out="bf16", group=None,
              stats=None, **mask) -> None:
    """The sharded wide tier for the listed rows (identical `rows` on every rank): writes their
    outputs and flags."""
    import torch.distributed as dist

    w = cuda.wide_partials(q, k, v, alpha, rows, stats=stats, max_row_keys=max_row_keys, **mask)
    gmax = w.maxv.clone()
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    cuda.rescale_wide_partials(w, gmax)
    dist.all_reduce(w.sumv, op=dist.ReduceOp.SUM, group=group)
    cuda.finalize_wide_partials(w, gmax, rows, out_tensor, flags, out=out, stats=stats)


def attention_kv_sharded(q, k, v, alpha, *, max_row_keys: int, out="bf16", group=None, stats=None,
                         parts: "cuda.Partials | None" = None, **mask):
    """Attention of every row of `q` over the union of all ranks' key ranges. `k`, `v` and
    `mask` (the `cuda.launch` mask keywords) describe this rank's range only; `max_row_keys`
    bounds a row's key count over all ranks. Returns (out bits, flags) on every rank.
    One host synchronisation per call: the count of rows for the wide tier (the same on every
    rank, so every rank takes the same collectives)."""
    parts = cuda.partials(q, k, v, alpha, parts=parts, stats=stats, max_row_keys=max_row_keys, **mask)
    merge_partials(parts, group)
    o, fl = cuda.finalize_partials(parts, max_row_keys, out=out, stats=stats)
    need = fl == 1
    if int(need.sum().item()):
        rows = need.nonzero().flatten()
        wide_tier(q, k, v, alpha, rows, o, fl, max_row_keys=max_row_keys, out=out, group=group, stats=stats, **mask)
    return o, fl
