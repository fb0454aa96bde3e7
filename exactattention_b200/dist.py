"""Long rows sharded by key range over ranks (one process per GPU), merged exactly.

Each rank holds a contiguous key range of every (sequence, kv head) and computes the row
partials of its range (`cuda.partials`): a reference exponent R and the fixed-point sums Z, N
with their error bounds. The merge is the split-KV combine of the reference's certified kernel
(triton_kernels.py:1081 `_ea_combine_kernel`; certified.py:213-246 `merge`), spread over ranks:

  1. one all-gather of every rank's flat partials (one message of rows x (24 + 20 dv) bytes per rank)
  2. on every rank, one kernel merges the gathered partials (MAX of the exponents, every partial
     re-expressed at them, SUM) and rounds every row (`cuda.merge_gathered`)

Rows whose merged interval does not certify (flag 1; the same rows on every rank, since every
rank merges the same integers) take the wide tier: each rank accumulates its keys of those rows
into 1536-bit windows (`cuda.wide_partials`), MAX all-reduce of the reference exponents, shift to
the maximum, SUM all-reduce of the 32-bit digits, certified rounding. With sync=True the count of
such rows is read on the host (one synchronisation; usually 0, so no wide-tier collectives run);
with sync=False a fixed-capacity wide tier runs every call with no host synchronisation (its unused
slots are empty), and rows beyond its capacity keep flag 1.

MAX and SUM are associative and commutative on integers, so the result is the same for every
rank count, rank order and reduction tree: the bits do not depend on how the keys were sharded.
The fixed-point headroom comes from the row's key count over ALL ranks (max_row_keys), so the
int64 sums cannot overflow.

`merge_partials` is the earlier two-collective form (MAX all-reduce, rescale, SUM all-reduce),
kept for callers that hold merged partials (it is what ea_merge_partials_nccl does in C).
"""

from __future__ import annotations

from . import cuda

WIDE_CAP = 2  # rows per call the sync-free mode finishes on the wide tier


def merge_partials(parts: "cuda.Partials", group=None, rescale=None) -> "cuda.Partials":
    """MAX all-reduce of (R, status, NR), rescale, SUM all-reduce of (Z, Zerr, N, Nerr), in place
    on `parts`. `rescale(parts, R_global, NR_global)` defaults to the device kernel; every rank must
    call this with the same row count and dv."""
    import torch.distributed as dist

    rows = parts.rows
    mx = parts.i32.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    (rescale or cuda.rescale_partials)(parts, mx[:rows], mx[2 * rows:].view(rows, parts.dv))
    parts.status.copy_(mx[rows:2 * rows])
    dist.all_reduce(parts.i64, op=dist.ReduceOp.SUM, group=group)
    return parts


def gather_partials(parts: "cuda.Partials", group=None):
    """Every rank's flat partials, concatenated in rank order on every rank: (buffer, world)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    g = parts.gathered(world)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(g, parts.flat, group=group)
    else:  # (CPU ranks in tests: gloo gathers into a list of views)
        dist.all_gather(list(g.view(world, -1).unbind(0)), parts.flat, group=group)
    return g, world


def wide_tier(q, k, v, alpha, rows, out_tensor, flags, *, max_row_keys: int, out="bf16", group=None,
              stats=None, **mask) -> None:
    """The sharded wide tier for the listed rows (identical `rows` on every rank; -1 marks an
    unused slot): writes their outputs and flags."""
    import torch.distributed as dist

    w = cuda.wide_partials(q, k, v, alpha, rows, stats=stats, max_row_keys=max_row_keys, **mask)
    gmax = w.maxv.clone()
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    cuda.rescale_wide_partials(w, gmax)
    dist.all_reduce(w.sumv, op=dist.ReduceOp.SUM, group=group)
    cuda.finalize_wide_partials(w, gmax, rows, out_tensor, flags, out=out, stats=stats)


def attention_kv_sharded(q, k, v, alpha, *, max_row_keys: int, out="bf16", group=None, stats=None,
                         parts: "cuda.Partials | None" = None, sync: bool = True, **mask):
    """Attention of every row of `q` over the union of all ranks' key ranges. `k`, `v` and
    `mask` (the `cuda.launch` mask keywords) describe this rank's range only; `max_row_keys`
    bounds a row's key count over all ranks. Returns (out bits, flags) on every rank.
    One collective per call (plus the wide tier's two when it runs). sync=True reads the count of
    wide-tier rows on the host; sync=False never synchronises (a fixed-capacity wide tier of
    WIDE_CAP rows runs every call; rows beyond it keep flag 1, which the caller sees in flags)."""
    parts = cuda.partials(q, k, v, alpha, parts=parts, stats=stats, max_row_keys=max_row_keys, **mask)
    g, world = gather_partials(parts, group)
    o, fl, wide_rows, wide_count = cuda.merge_gathered(g, world, parts, max_row_keys, out=out, stats=stats)
    if sync:
        n = int(wide_count.item())
        if n:
            wide_tier(q, k, v, alpha, wide_rows[:n], o, fl, max_row_keys=max_row_keys, out=out, group=group,
                      stats=stats, **mask)
    else:
        # the list is in row order and padded with -1, so its first WIDE_CAP slots are the same on
        # every rank
        wide_tier(q, k, v, alpha, wide_rows[:min(WIDE_CAP, parts.rows)], o, fl, max_row_keys=max_row_keys, out=out,
                  group=group, stats=stats, **mask)
    return o, fl
