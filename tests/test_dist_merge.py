"""KV-range sharding: the collective choreography of dist.merge_partials on CPU ranks (gloo).

The device rescale kernel is replaced by `np_rescale`, its restatement in numpy (the floor shift
and error growth of ea_numerics.h `rescale`), so these tests need no GPU. They check that the
merged partials are the same on every rank, equal a sequential max-then-sum merge of all ranks'
partials, and do not depend on the rank count or order. The numerics of the merged result are
checked against the oracle by the GPU tests (test_gpu_parity.py, kv-sharded cases).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from exactattention_b200 import cuda, dist as ea_dist

R_EMPTY = np.iinfo(np.int32).min


def _rescale_np(acc: np.ndarray, err: np.ndarray, s: np.ndarray):
    acc, err, s = acc.astype(np.int64), err.astype(np.uint64), s.astype(np.int64)
    out_a, out_e = acc.copy(), err.copy()
    for i in np.flatnonzero(s > 0):
        a, e, sh = int(acc.flat[i]), int(err.flat[i]), int(s.flat[i])
        if sh >= 63:
            na, lost = (-1 if a < 0 else 0), int(a != 0)
        else:
            na = a >> sh
            lost = int((na << sh) != a)
        ne = int(e != 0) if sh >= 64 else (e >> sh) + int(e & ((1 << sh) - 1) != 0)
        out_a.flat[i], out_e.flat[i] = na, np.uint64(ne + lost)
    return out_a, out_e


def np_rescale(parts, R_g, NR_g):
    """numpy restatement of partials_rescale_kernel: empty partials become zeros; the others are
    floor-shifted to the global exponent."""
    R, Rg = parts.R.numpy(), R_g.numpy()
    NR, NRg = parts.NR.numpy(), NR_g.numpy()
    Z, Ze = parts.Z.numpy(), parts.Zerr.numpy().view(np.uint64)
    N, Ne = parts.N.numpy(), parts.Nerr.numpy().view(np.uint64)
    for acc, err, e, g in ((Z, Ze, R, Rg), (N, Ne, NR, NRg)):
        empty = e == R_EMPTY
        s = np.where(empty | (g == R_EMPTY), 0, g.astype(np.int64) - e.astype(np.int64))
        a2, e2 = _rescale_np(acc, err, s)
        a2[empty], e2[empty] = 0, 0
        acc[...], err[...] = a2, e2
    parts.R.copy_(torch.from_numpy(Rg.copy()))
    parts.NR.copy_(torch.from_numpy(NRg.copy()))


def make_parts(seed: int, rows: int, dv: int) -> cuda.Partials:
    """Random partials in the ranges tier 1 produces (|Z|, |N| < 2^58, exponents within 40)."""
    rng = np.random.default_rng(seed)
    p = cuda.Partials(rows, dv, "cpu")
    R = rng.integers(-40, 40, rows).astype(np.int32)
    R[rng.random(rows) < 0.2] = R_EMPTY
    p.R.copy_(torch.from_numpy(R))
    p.status.copy_(torch.from_numpy(np.where(rng.random(rows) < 0.1, 1, 0).astype(np.int32)))
    p.Z.copy_(torch.from_numpy(np.where(R == R_EMPTY, 0, rng.integers(0, 1 << 58, rows))))
    p.Zerr.copy_(torch.from_numpy(np.where(R == R_EMPTY, 0, rng.integers(0, 64, rows))))
    NR = (R[:, None] + rng.integers(-3, 4, (rows, dv))).astype(np.int32)
    NR[R == R_EMPTY] = R_EMPTY
    NR[rng.random((rows, dv)) < 0.05] = R_EMPTY
    p.NR.copy_(torch.from_numpy(NR))
    p.N.copy_(torch.from_numpy(np.where(NR == R_EMPTY, 0, rng.integers(-(1 << 58), 1 << 58, (rows, dv)))))
    p.Nerr.copy_(torch.from_numpy(np.where(NR == R_EMPTY, 0, rng.integers(0, 64, (rows, dv)))))
    return p


def sequential_merge(all_parts):
    """max of exponents and status, rescale each, sum: the merge on one process."""
    R_g = torch.stack([p.R for p in all_parts]).max(0).values
    NR_g = torch.stack([p.NR for p in all_parts]).max(0).values
    st = torch.stack([p.status for p in all_parts]).max(0).values
    for p in all_parts:
        np_rescale(p, R_g, NR_g)
    out = all_parts[0]
    for p in all_parts[1:]:
        out.i64 += p.i64
    out.status.copy_(st)
    return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, rows: int, dv: int, seeds, result_dir: str):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = make_parts(seeds[rank], rows, dv)
        ea_dist.merge_partials(p, rescale=np_rescale)
        np.save(os.path.join(result_dir, f"i32_{rank}.npy"), p.i32.numpy())
        np.save(os.path.join(result_dir, f"i64_{rank}.npy"), p.i64.numpy())
    finally:
        dist.destroy_process_group()


def _run(world: int, rows: int, dv: int, seeds, tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(world, _free_port(), rows, dv, seeds, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    i32 = [np.load(tmp_path / f"i32_{r}.npy") for r in range(world)]
    i64 = [np.load(tmp_path / f"i64_{r}.npy") for r in range(world)]
    return i32, i64


@pytest.mark.parametrize("world", [2, 3])
def test_merge_matches_sequential(world, tmp_path):
    rows, dv = 37, 16
    seeds = [100 + r for r in range(world)]
    i32, i64 = _run(world, rows, dv, seeds, tmp_path)
    for r in range(1, world):
        assert np.array_equal(i32[0], i32[r]) and np.array_equal(i64[0], i64[r])
    ref = sequential_merge([make_parts(s, rows, dv) for s in seeds])
    assert np.array_equal(i32[0], ref.i32.numpy())
    assert np.array_equal(i64[0], ref.i64.numpy())


def test_merge_is_order_free(tmp_path):
    rows, dv = 29, 8
    seeds = [7, 8, 9]
    a = sequential_merge([make_parts(s, rows, dv) for s in seeds])
    b = sequential_merge([make_parts(s, rows, dv) for s in reversed(seeds)])
    assert np.array_equal(a.i32.numpy(), b.i32.numpy()) and np.array_equal(a.i64.numpy(), b.i64.numpy())
    (tmp_path / "rev").mkdir()
    i32, i64 = _run(3, rows, dv, list(reversed(seeds)), tmp_path / "rev")
    assert np.array_equal(i32[0], a.i32.numpy()) and np.array_equal(i64[0], a.i64.numpy())


def test_merge_single_rank_is_identity_up_to_rescale():
    p = make_parts(3, 11, 4)
    before = p.i64.clone()
    sequential_merge([p])
    assert torch.equal(p.i64, before)


def _gather_worker(rank: int, world: int, port: int, rows: int, dv: int, seeds, result_dir: str):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = make_parts(seeds[rank], rows, dv)
        g, w = ea_dist.gather_partials(p)
        assert w == world
        np.save(os.path.join(result_dir, f"g_{rank}.npy"), g.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_is_every_flat_buffer_in_rank_order(world, tmp_path):
    """The one-collective merge's gather: every rank holds every rank's flat partials in rank
    order, in the flat layout (the merge kernel then reads rank s's fields at s x the flat size),
    and merging them gives the same partials as the MAX / rescale / SUM form."""
    import torch.multiprocessing as mp

    rows, dv = 23, 8
    seeds = [300 + r for r in range(world)]
    mp.start_processes(_gather_worker, args=(world, _free_port(), rows, dv, seeds, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    gs = [np.load(tmp_path / f"g_{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(gs[0], gs[r])
    flat = np.concatenate([make_parts(s, rows, dv).flat.numpy() for s in seeds])
    assert np.array_equal(gs[0], flat)
    # the layout: rank s's partials read back from its slice of the gathered buffer
    n_flat = make_parts(seeds[0], rows, dv).flat.numel()
    views = []
    for s in range(world):
        p = cuda.Partials(rows, dv, "cpu")
        p.flat.copy_(torch.from_numpy(gs[0][s * n_flat:(s + 1) * n_flat]))
        views.append(p)
    merged = sequential_merge(views)
    ref = sequential_merge([make_parts(s, rows, dv) for s in seeds])
    assert np.array_equal(merged.i32.numpy(), ref.i32.numpy()) and np.array_equal(merged.i64.numpy(), ref.i64.numpy())


def test_flat_layout_matches_header():
    """The flat buffer's size is EA_PARTIALS_FLAT_BYTES(rows, dv) of include/exactattn_cuda.h."""
    for rows, dv in ((1, 1), (7, 3), (64, 128), (5, 256)):
        p = cuda.Partials(rows, dv, "cpu")
        want = (rows * (16 + 16 * dv) + rows * (8 + 4 * dv) + 7) & ~7
        assert p.flat.numel() * 8 == want
        assert p.R.data_ptr() - p.flat.data_ptr() == 8 * rows * (2 + 2 * dv)
