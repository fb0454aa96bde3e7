"""KV-range sharding over real ranks: one process per GPU, NCCL all-reduces (B200, >= 2 GPUs).

Every rank holds a contiguous key range; dist.attention_kv_sharded must return, on every rank,
the bits one single-GPU launch gives over all keys. Skipped when the box has one GPU.
"""

import os
from datetime import timedelta

import numpy as np
import pytest

from gen import bf16

pytestmark = pytest.mark.gpu


def _store(result_dir: str) -> str:
    # a file rendezvous in the test's own directory: no TCP port to race other processes for
    return "file://" + os.path.join(result_dir, "pg_store")


def _case(d=128):
    rng = np.random.default_rng(515)
    rows, n = 32, 6000
    Q, K, V = bf16(rng, (rows, d), "outlier"), bf16(rng, (n, d), "outlier"), bf16(rng, (n, d), "wide")
    kl = rng.integers(n // 2, n + 1, rows).astype(np.int64)
    return Q, K, V, kl


def _worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    import exactattention_b200 as ea
    from exactattention_b200 import dist as ea_dist

    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=_store(result_dir), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        Q, K, V, kl = _case()
        n = K.shape[0]
        lo, hi = n * rank // world, n * (rank + 1) // world
        t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
        klen = np.clip(kl - lo, 0, hi - lo).astype(np.int64)
        out, flags = ea_dist.attention_kv_sharded(t(Q), t(K[lo:hi]), t(V[lo:hi]), ea.default_alpha(128),
                                                  max_row_keys=n, kv_base=t(np.zeros_like(kl)), kv_len=t(klen))
        torch.cuda.synchronize(dev)
        np.save(os.path.join(result_dir, f"out_{rank}.npy"), out.cpu().numpy())
        np.save(os.path.join(result_dir, f"flags_{rank}.npy"), flags.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_nccl_kv_sharded_matches_single_gpu(world, tmp_path):
    import torch
    import torch.multiprocessing as mp

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, 0, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    Q, K, V, kl = _case()
    dev = torch.device("cuda", 0)
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    full, fflags = cuda.launch(t(Q), t(K), t(V), ea.default_alpha(128), kv_base=t(np.zeros_like(kl)), kv_len=t(kl))
    full = full.cpu().numpy()
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"flags_{r}.npy"), fflags.cpu().numpy()), r
        assert np.array_equal(np.load(tmp_path / f"out_{r}.npy"), full), r


def _c5_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    from exactattention_b200 import dist as ea_dist, workloads as w

    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=_store(result_dir), rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=dev)
    try:
        case = w.device_case("c5", dev, shard=rank, nshards=world)
        kw = dict(case["kw"])
        mrk = kw.pop("max_row_keys")
        for sync in (True, False):  # host-read wide-row count / fixed-capacity wide tier, no host sync
            out, flags = ea_dist.attention_kv_sharded(case["q"], case["k"], case["v"], case["cfg"].alpha,
                                                      max_row_keys=mrk, splits=32, sync=sync, **kw)
            torch.cuda.synchronize(dev)
            np.save(os.path.join(result_dir, f"c5_out_{rank}_{int(sync)}.npy"), out.cpu().numpy())
            np.save(os.path.join(result_dir, f"c5_flags_{rank}_{int(sync)}.npy"), flags.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_nccl_c5_sharded_sha(tmp_path):
    """Config 5 sharded by key range over the ranks: every rank's merged output has the
    reference's SHA-256 (the bits do not depend on the GPU count)."""
    import hashlib
    import json

    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    gold = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "configs.json"))).get("c5")
    if gold is None:
        pytest.skip("no golden SHA for c5")
    mp.start_processes(_c5_worker, args=(world, 0, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        for sync in (1, 0):
            assert not np.load(tmp_path / f"c5_flags_{r}_{sync}.npy").any()
            out = np.load(tmp_path / f"c5_out_{r}_{sync}.npy").view(np.uint16)
            assert hashlib.sha256(np.ascontiguousarray(out).tobytes()).hexdigest() == gold, (r, sync)


def _raw_comm_worker(rank, world, port, result_dir):
    """ea_merge_partials_nccl on a communicator made directly with NCCL's C API (as a C / C++
    server would hold one), the unique id exchanged through the process group's store; the same
    partials merged by dist.merge_partials (torch.distributed) must come out bit for bit equal."""
    import ctypes

    import torch
    import torch.distributed as dist

    import exactattention_b200 as ea
    from exactattention_b200 import cuda, dist as ea_dist

    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=_store(result_dir), rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    nccl = ctypes.CDLL("libnccl.so.2")

    class UniqueId(ctypes.Structure):
        _fields_ = [("internal", ctypes.c_byte * 128)]

    uid = UniqueId()
    idt = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        assert nccl.ncclGetUniqueId(ctypes.byref(uid)) == 0
        idt.copy_(torch.frombuffer(bytearray(ctypes.string_at(ctypes.addressof(uid), 128)), dtype=torch.uint8))
    dist.broadcast(idt, 0)
    ctypes.memmove(ctypes.addressof(uid), bytes(idt.cpu().numpy().tobytes()), 128)
    comm = ctypes.c_void_p()
    nccl.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, UniqueId, ctypes.c_int]
    assert nccl.ncclCommInitRank(ctypes.byref(comm), world, uid, rank) == 0
    try:
        Q, K, V, kl = _case()
        n = K.shape[0]
        lo, hi = n * rank // world, n * (rank + 1) // world
        t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
        klen = np.clip(kl - lo, 0, hi - lo).astype(np.int64)
        args = (t(Q), t(K[lo:hi]), t(V[lo:hi]), ea.default_alpha(128))
        mask = dict(kv_base=t(np.zeros_like(kl)), kv_len=t(klen))
        pa = cuda.partials(*args, max_row_keys=n, **mask)
        pb = cuda.partials(*args, max_row_keys=n, **mask)
        ea_dist.merge_partials(pa)
        cuda.merge_partials_nccl(pb, comm.value)
        torch.cuda.synchronize(dev)
        same = torch.equal(pa.i32, pb.i32) and torch.equal(pa.i64, pb.i64)
        oa, fa = cuda.finalize_partials(pa, n)
        ob, fb = cuda.finalize_partials(pb, n)
        torch.cuda.synchronize(dev)
        same = same and torch.equal(oa, ob) and torch.equal(fa, fb)
        np.save(os.path.join(result_dir, f"raw_same_{rank}.npy"), np.array([same]))
        dist.barrier()
    finally:
        nccl.ncclCommDestroy(comm)
        dist.destroy_process_group()


def test_merge_partials_nccl_raw_communicator(tmp_path):
    """The C-ABI merge over a raw NCCL communicator equals the torch.distributed merge."""
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_raw_comm_worker, args=(world, 0, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        assert bool(np.load(tmp_path / f"raw_same_{r}.npy")[0]), r
