"""Benchmark of certified ExactAttention on B200: certified QK pairs/s and decode tokens/s.

python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5|c2|c3|c4] [--extras c2,c3,c4|none]
               [--splits S] [--impl ours|reference] [--no-e2e] [--no-cpu]

The headline (`value`) is config 5: batch 4 x 16 q / 8 kv heads x one query token against 2^20
keys (67,108,864 certified pairs per step). On one GPU it is the whole job; under torchrun every
(sequence, kv head) is sharded by key range over the ranks, one NCCL all-gather brings every rank
all ranks' int64 row partials, and one kernel merges them exactly (MAX of the exponents, SUM of
the rescaled integers) and rounds: strong scaling, the same bits at every N. In the same run configs 2, 3 and 4 are measured into `extra.configs` (at
N > 1 sharded by (sequence, kv head) segments: every rank a contiguous share of the rows, no
data-path collective, outputs gathered for the hash). Every config's output is hashed (SHA-256 of
the bf16 bits in canonical row order) and compared with tests/golden/configs.json (`sha_ok`).

  value         c5 pairs/s of the whole job, inputs resident in HBM; CUDA events around each step
                on the launch stream, L2 flushed (a 256 MiB write) between steps; max over ranks
  e2e           the same metric through the public API from pinned host buffers: one GPU
                ea_attention_cuda_ranges (host pointers); N GPUs each rank's key shard copied in,
                the sharded call, the outputs copied out; inside the timed region
  roofline      the hot (tier-1) kernel, timed live with CUDA events on the launch stream
                (ea_kernel_timing): decode (c3, c5) against HBM at 512 bytes of K and V per
                (kv head, key) plus q, outputs and page-table entries; prefill (c2, c4) against
                the int8 tensor-core roofline at 7,936 int8 ops per pair (the reference's 4 x 4
                score and 5 x 3 P.V slice plan)
  cpu_baseline  the reference's C++ certified kernel (oracle/_ref) on whole (sequence, kv head)
                segments of the same config, several at once on the host's cores (rank 0, N = 1)
`--impl reference` times only that CPU implementation, on the same config and metric.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

INT8_OPS_PER_PAIR = 7936        # QK 4x4 slices + P.V 5x3 slices at d = 128 (the reference's slice plan)
BF16_EQUIV_FLOPS_PER_PAIR = 512  # 4 d
KV_BYTES_PER_KEY = 512           # bf16 K and V rows of d = 128 for one kv head, read once
HOT_KERNEL = {"c2": "tc_prefill_kernel", "c3": "tc_decode_kernel", "c4": "tc_prefill_kernel",
              "c5": "tc_decode_kernel"}
DEFAULT_SPLITS = {"c2": 1, "c3": 8, "c4": 1, "c5": 32}
# our kernel launches per step: tier 1, split combine / list kernel, and the fallback tiers'
# fixed launches (they run on device-side counts, so they launch every step); KV-sharded c5: the
# decode kernel, the split combine (export), the gathered merge, and the fixed-capacity wide tier
# (wide partials, rescale, finalize; empty slots)
LAUNCHES = {"c2": 9, "c3": 10, "c4": 11, "c5": 10, "c5-sharded": 7}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c5", choices=["c2", "c3", "c4", "c5"])
    ap.add_argument("--extras", default="c2,c3,c4", help="configs also measured in the same run, or 'none'")
    ap.add_argument("--splits", type=int, default=0, help="KV splits of the headline config (0: its default)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--kv-shard", default="", help="c5 on one GPU: only key range K of N (\"K/N\"), the share of "
                    "one rank of an N-GPU run (a smaller case of the same kernel, for profiling)")
    ap.add_argument("--seqs", type=int, default=0, help="c3 / c4 on one GPU: only the first SEQS sequences (a smaller "
                    "case of the same kernels, for profiling)")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def golden() -> dict:
    p = os.path.join(ROOT, "tests", "golden", "configs.json")
    return json.load(open(p)) if os.path.exists(p) else {}


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.t.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if len(r) >= 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 8 for i in range(4) if r[4 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's C++ kernel on whole (sequence, kv head) segments
# ---------------------------------------------------------------------------

_SEGMENTS: dict = {}
# c5's 2^20-key segments take the reference kernel ~15 s each on two threads: its sample is the
# first 2^18 keys of each segment (one rank's key range at N = 4)
SAMPLE_KEYS = {"c5": 1 << 18}


def cpu_segments(name: str, count: int):
    """The first `count` (sequence, kv head) segments of a config, c5's cut to SAMPLE_KEYS keys
    (made once, reused by every step; the host generator makes a 2^20-key tensor in under a
    second)."""
    from exactattention_b200 import workloads

    key = (name, count)
    if key not in _SEGMENTS:
        cfg = workloads.config(name)
        segs = []
        for seg in workloads.segments(cfg):
            n = SAMPLE_KEYS.get(name)
            if n:
                b, kvh, Q, K, V, rp, ki, canon = seg
                rows = Q.shape[0]
                rp = np.arange(rows + 1, dtype=np.int64) * n
                ki = np.tile(np.arange(n, dtype=np.int64), rows)
                seg = (b, kvh, Q, np.ascontiguousarray(K[:n]), np.ascontiguousarray(V[:n]), rp, ki, canon)
            segs.append(seg)
            if len(segs) == count:
                break
        _SEGMENTS[key] = (cfg, segs)
    return _SEGMENTS[key]


def cpu_reference_step(name: str, cores: int):
    """One step of the reference kernel: as many segments at once as the cores allow, each call on
    as many threads as the segment has rows (the kernel parallelises over rows). Returns
    (pairs, seconds, segments, threads used, flagged rows)."""
    from oracle import ref

    per = {"c2": None, "c3": 2, "c4": None, "c5": 2}[name]  # rows per segment (prefill: all cores)
    if per is None:
        conc, threads = 1, cores
    else:
        conc, threads = max(1, min(cores // per, 16)), per  # ~0.6 GB of host memory per sampled segment
    cfg, segs = cpu_segments(name, conc)

    def one(seg):
        _, _, Q, K, V, rp, ki, _ = seg
        _, fl = ref.attention_ref(Q, K, V, cfg.alpha, rp, ki, threads=threads, splits=1, tile=64, fallback=False)
        return int(rp[-1]), int((fl != 0).sum())

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=conc) as ex:
        res = list(ex.map(one, segs))
    secs = time.perf_counter() - t0
    return sum(p for p, _ in res), secs, len(segs), conc * threads, sum(f for _, f in res)


def cpu_sample_desc(name, segs, threads, pairs, secs, flagged):
    from oracle import ref

    what = (f"the first {SAMPLE_KEYS[name]} keys of {segs} (sequence, kv head) segment(s)" if name in SAMPLE_KEYS
            else f"{segs} whole (sequence, kv head) segment(s)")
    return (f"{what} of {name} per step, run at once on {threads} threads (host: {os.cpu_count()} logical CPUs); "
            f"{pairs} pairs in {secs:.2f} s; "
            f"{flagged} rows flagged 1 (the C++ kernel's own fallback count); the reference kernel built for "
            f"{ref.build_variant()}")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import ref

    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libexactattn_cpu.so not built"}))
        return
    from exactattention_b200 import workloads

    cfg = workloads.config(args.config)
    cores = os.cpu_count() or 1
    for _ in range(max(1, args.warmup)):
        cpu_reference_step(args.config, cores)
    tot_p, tot_s = 0, 0.0
    for _ in range(args.steps):
        p, s, n, threads, flagged = cpu_reference_step(args.config, cores)
        tot_p += p
        tot_s += s
    v = tot_p / tot_s
    sample = cpu_sample_desc(args.config, n, threads, tot_p // args.steps, tot_s / args.steps, flagged)
    print(json.dumps({
        "impl": "reference", "metric": "certified QK pairs/s", "value": v, "unit": "pairs/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * tot_s / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "config": {"workload": args.config, "job_pairs": cfg.pairs, "rows": cfg.rows},
        "cpu_baseline": {"value": v, "unit": "pairs/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": v, "unit": "pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---------------------------------------------------------------------------
# GPU cases: the rank's share of a config
# ---------------------------------------------------------------------------

def row_share(name: str, cfg, rank: int, world: int) -> tuple[int, int]:
    """Contiguous rows [r0, r1) of this rank when c2 / c3 / c4 are sharded by (sequence, kv head):
    c2 by kv head (its GQA pair of q heads), c3 and c4 by sequence."""
    from exactattention_b200 import workloads as w

    if name == "c2":
        g0, g1 = w.HKV * rank // world, w.HKV * (rank + 1) // world
        return g0 * w.GROUP * cfg.q_tokens, g1 * w.GROUP * cfg.q_tokens
    per = w.HQ * cfg.q_tokens  # rows per sequence
    b0, b1 = cfg.batch * rank // world, cfg.batch * (rank + 1) // world
    return b0 * per, b1 * per


def slice_case(name: str, case: dict, r0: int, r1: int) -> dict:
    """The case restricted to rows [r0, r1) (a sequence- or kv-head-aligned range)."""
    import torch

    from exactattention_b200 import cuda, workloads as w

    kw = dict(case["kw"])
    dev = case["q"].device
    q = case["q"][r0:r1]
    if name == "c3":
        b0, b1 = r0 // w.HQ, r1 // w.HQ
        kw["page_table"] = kw["page_table"][b0:b1].contiguous()
        kw["seq_lens"] = kw["seq_lens"][b0:b1].contiguous()
    else:
        kb = kw["kv_base"][r0:r1].contiguous()
        kl = kw["kv_len"][r0:r1].contiguous()
        kw["kv_base"], kw["kv_len"] = kb, kl
        kbn, kln = kb.cpu().numpy(), kl.cpu().numpy()
        if "blocks" in kw:
            kw["blocks"] = torch.from_numpy(cuda.row_blocks(kbn, kln)).to(dev)
        if "segments" in kw:
            kw["segments"] = torch.from_numpy(cuda.row_segments(kbn)).to(dev)
        if "row_ptr" in kw:
            rp = kw["row_ptr"]
            a, b = int(rp[r0].item()), int(rp[r1].item())
            kw["row_ptr"] = (rp[r0:r1 + 1] - a).contiguous()
            kw["key_idx"] = kw["key_idx"][a:b].contiguous()
    return dict(cfg=case["cfg"], q=q.contiguous(), k=case["k"], v=case["v"], kw=kw)


def algorithmic(name: str, cfg, rows: int, keys_per_row_sum: int | None = None, kv_keys: int | None = None,
                extra_bytes: int = 0) -> dict:
    """The hot kernel's algorithmic work per launch on this rank: int8 tensor ops for the prefill
    shapes (pairs on the tensor cores x 7,936), HBM bytes for decode (K + V of every (segment,
    visible key) once, q, outputs, page-table entries)."""
    if name in ("c2", "c4"):
        return {"bound": "tensor", "units": keys_per_row_sum * INT8_OPS_PER_PAIR, "what": "int8 ops",
                "per_unit": f"{INT8_OPS_PER_PAIR} int8 ops per (row, key) pair on the tensor cores"}
    b = kv_keys * KV_BYTES_PER_KEY + rows * 2 * 128 * 2 + extra_bytes
    return {"bound": "hbm", "units": b, "what": "bytes",
            "per_unit": f"{KV_BYTES_PER_KEY} B of bf16 K and V per (kv head, key) + q, out, page-table bytes"}


def roofline(alg: dict, kernel_ms: float, pk: dict, kern: str, launches: int, traffic) -> dict:
    if alg["bound"] == "tensor":
        # dense int8 = 2x dense bf16 on B200 (the nominal ratio applied to the measured bf16 GEMM)
        peak, unit = 2.0 * pk["bf16_tflops"], "TOPS(int8)"
        achieved = alg["units"] / (kernel_ms / 1000.0) / 1e12
        src = f"2 x {pk['source']} bf16 {pk['bf16_tflops']} TFLOP/s (no int8 peak measured)"
    else:
        peak, unit = pk["hbm_gbs"], "GB/s"
        achieved = alg["units"] / (kernel_ms / 1000.0) / 1e9
        src = f"{pk['source']} HBM copy {pk['hbm_gbs']} GB/s"
    return {"bound": alg["bound"], "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": traffic, "kernel": kern, "kernel_ms": kernel_ms, "kernel_launches_timed": launches,
            "algorithmic_per_launch": alg["units"], "algorithmic_unit": alg["what"],
            "algorithmic_per_unit": alg["per_unit"], "peak_source": src}


def profile_traffic(kern: str, name: str):
    p = os.path.join(ROOT, "profiles", f"{kern}_{name}.json")
    return json.load(open(p)).get("dram_bytes_per_launch") if os.path.exists(p) else None


class Runner:
    """One process per GPU; the collective plumbing of the run."""

    def __init__(self):
        import torch
        import torch.distributed as dist

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = torch.device("cuda", self.local)
        torch.cuda.set_device(self.dev)
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=self.dev)
        self.dist = dist
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        import torch

        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather_rows(self, out, total_rows: int):
        """Every rank's contiguous output rows, concatenated in rank order (rank 0 gets the whole
        output; padded to equal shares for all_gather)."""
        import torch

        if self.world == 1:
            return out
        n = torch.tensor([out.shape[0]], dtype=torch.int64, device=self.dev)
        ns = [torch.zeros_like(n) for _ in range(self.world)]
        self.dist.all_gather(ns, n)
        ns = [int(x.item()) for x in ns]
        m = max(ns)
        b = out.contiguous().view(torch.uint8)  # NCCL moves bytes (it has no 16-bit integer type)
        pad = torch.zeros((m, b.shape[1]), dtype=torch.uint8, device=self.dev)
        pad[:b.shape[0]] = b
        allp = torch.empty((self.world * m, b.shape[1]), dtype=torch.uint8, device=self.dev)
        self.dist.all_gather_into_tensor(allp, pad)
        full = torch.cat([allp[i * m:i * m + ns[i]] for i in range(self.world)]).view(out.dtype)
        assert full.shape[0] == total_rows
        return full

    def time_steps(self, step, steps: int, warmup: int, clocks: bool = False):
        """W untimed steps, then K steps bracketed by barrier + synchronize, each timed with CUDA
        events on the launch stream after an L2 flush; returns (max-over-ranks mean ms, hot-kernel
        ms per launch or None, launches timed, clock record)."""
        import torch

        from exactattention_b200 import cuda

        for _ in range(max(3, warmup)):
            step()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream(self.dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        cuda.kernel_timing(1)
        clk = Clocks(self.local) if clocks else None
        if clk:
            clk.start()
        self.barrier()
        torch.cuda.synchronize()
        for i in range(steps):
            self.flush.fill_(i & 0xFF)
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        self.barrier()
        rec = clk.stop() if clk else None
        k_tot, k_n = cuda.kernel_timing(2)
        cuda.kernel_timing(0)
        ms = sum(a.elapsed_time(b) for a, b in ev) / steps
        return self.max(ms), (k_tot / k_n if k_n else None), k_n, rec


def config_splits(name: str, case: dict, sms: int) -> int:
    """KV splits of a config's rank share: c4's prefix blocks (128 rows each) are too few to fill
    the GPU, so each takes enough KV splits for about 1.5 waves; the others use their measured
    best (c2 1, c3 8, c5 32)."""
    if name == "c4":
        nb = int(case["kw"]["blocks"].shape[0])
        return max(1, -(-3 * sms // (2 * nb)))
    return DEFAULT_SPLITS[name]


def run_config(R: Runner, name: str, args, headline: bool) -> dict:
    """Measures one config on this rank (its share at N > 1); returns the config's record (rank 0
    fills in the hash check)."""
    import torch

    from exactattention_b200 import cuda, workloads

    world, rank = R.world, R.rank
    # c5 at N > 1: KV-range shards merged over NCCL. --kv-shard K/N on one GPU: only that key range
    # of every segment, through the single-GPU launch (a smaller case of the same kernel, e.g. for a
    # profile; no merge, no hash check)
    kv_sharded = name == "c5" and world > 1
    one_shard = name == "c5" and world == 1 and bool(args.kv_shard) and headline
    ks, kn = rank, world
    if one_shard:
        ks, kn = (int(x) for x in args.kv_shard.split("/"))
    if name == "c5":
        case = workloads.device_case(name, R.dev, shard=ks, nshards=kn) if (kv_sharded or one_shard) else \
            workloads.device_case(name, R.dev)
        r0, r1 = 0, case["cfg"].rows
    else:
        full = workloads.device_case(name, R.dev)
        r0, r1 = row_share(name, full["cfg"], rank, world)
        if headline and args.seqs and name in ("c3", "c4") and world == 1:
            r0, r1 = 0, args.seqs * workloads.HQ * full["cfg"].q_tokens
        case = slice_case(name, full, r0, r1) if (r0, r1) != (0, full["cfg"].rows) else full
        del full
    cfg = case["cfg"]
    q, k, v, kw = case["q"], case["k"], case["v"], case["kw"]
    rows = q.shape[0]
    sms = torch.cuda.get_device_properties(R.dev).multi_processor_count
    splits = (args.splits if headline and args.splits else 0) or config_splits(name, case, sms)
    stats = cuda.new_stats(R.dev)
    cuda.reserve_workspace(rows, splits, 128)
    out = torch.empty((rows, 128), dtype=torch.int16, device=R.dev)
    flags = torch.empty(rows, dtype=torch.uint8, device=R.dev)

    if kv_sharded:
        from exactattention_b200 import dist as ea_dist

        parts = cuda.Partials(rows, 128, R.dev)
        kwl = dict(kw)
        mrk = kwl.pop("max_row_keys")

        def step():
            o, f = ea_dist.attention_kv_sharded(q, k, v, cfg.alpha, max_row_keys=mrk, splits=splits, stats=stats,
                                                parts=parts, sync=False, **kwl)
            out.copy_(o)
            flags.copy_(f)
    else:
        def step():
            cuda.launch(q, k, v, cfg.alpha, splits=splits, out_tensor=out, flags=flags, stats=stats, **kw)

    step()
    torch.cuda.synchronize()
    stats.zero_()
    ms, kernel_ms, k_n, clk = R.time_steps(step, args.steps, args.warmup, clocks=headline)
    st = stats.cpu().numpy() // max(1, args.steps + max(3, args.warmup))  # per step (every step counts)
    ok_local = bool(not flags.any().item())
    ok = R.max(0.0 if ok_local else 1.0) == 0.0

    # the job's output in canonical row order, hashed on rank 0
    if name == "c5" or (headline and args.seqs):
        full_out = out  # c5: every rank holds every row after the merge
    else:
        full_out = R.gather_rows(out, cfg.rows)
    sha = hashlib.sha256(full_out.cpu().numpy().view(np.uint16).tobytes()).hexdigest() if rank == 0 else None
    gold = golden().get(name)

    # algorithmic work of this rank's hot-kernel launch
    if name == "c3":
        ctx = kw["seq_lens"].cpu().numpy().astype(np.int64)
        alg = algorithmic(name, cfg, rows, kv_keys=int(ctx.sum()) * workloads.HKV,
                          extra_bytes=int(((ctx + cfg.page_size - 1) // cfg.page_size).sum()) * workloads.HKV * 4)
    elif name == "c5":
        keys = int(kw["kv_len"].cpu().numpy()[::workloads.GROUP].sum())  # one per (sequence, kv head)
        alg = algorithmic(name, cfg, rows, kv_keys=keys)
    else:
        alg = algorithmic(name, cfg, rows, keys_per_row_sum=int(kw["kv_len"].sum().item()))
    kern = HOT_KERNEL[name]
    rl = roofline(alg, kernel_ms if kernel_ms else ms, peaks(), kern, k_n, profile_traffic(kern, name))
    job_pairs = cfg.pairs if not args.kv_shard else cfg.pairs // kn
    partial_job = bool(args.kv_shard) or (headline and bool(args.seqs))
    if headline and args.seqs:
        job_pairs = int(cfg.row_keys()[:rows].sum())  # the first rows in canonical order
    tokens = cfg.rows if name in ("c3", "c5") else None  # decode: one query token per (sequence, q head) row
    rec = {
        "value": job_pairs / (ms / 1000.0), "unit": "pairs/s", "ms_per_step": ms, "job_pairs": job_pairs,
        "rows": cfg.rows, "rows_per_rank": rows, "splits": splits,
        "parallelism": (f"kv-range shards x{world}, one NCCL all-gather of the int64 partials, exact merge" if kv_sharded and world > 1 else
                        f"(sequence, kv head) shards x{world}, outputs gathered for the hash" if world > 1 else
                        "1 GPU"),
        "decode_tokens_per_s": (tokens / (ms / 1000.0)) if tokens else None,
        "query_rows_per_s": cfg.rows / (ms / 1000.0),
        "roofline": rl,
        "flags_all_zero": ok, "sha256": sha, "sha_ok": (sha == gold) if (rank == 0 and gold and not partial_job) else None,
        "certified_per_step": {"tier1_uncertified_rows": int(st[2]), "tier2_uncertified_rows": int(st[9]),
                               "tier2_pairs": int(st[10]), "domain_rows": int(st[3]), "unresolved_rows": int(st[4]),
                               "waits_expired": int(st[8]), "host_fallbacks": int(st[6]),
                               "tensor_core_pairs": int(st[7]), "score_exact": int(st[0]),
                               "weight_wide": int(st[1])},
        "clocks": clk,
        "launches_per_step": LAUNCHES["c5-sharded" if kv_sharded else name],
    }
    if headline and not args.no_e2e and not partial_job:
        rec["e2e"] = e2e(R, name, case, splits, out, kv_sharded, job_pairs)
    del case, q, k, v, kw
    torch.cuda.empty_cache()
    return rec


def e2e(R: Runner, name: str, case: dict, splits: int, out_dev, kv_sharded: bool, job_pairs: int) -> dict:
    """The same metric end to end from pinned host buffers, through the public API: one GPU the
    host-pointer C ABI (ea_attention_cuda_ranges / _paged / the CSR entry), N GPUs the rank's
    shard copied in (q, K, V, masks), dist.attention_kv_sharded, the outputs copied out. Wall
    clock around K calls after a barrier, max over ranks."""
    import torch

    from exactattention_b200 import cuda

    cfg, q, k, v, kw = case["cfg"], case["q"], case["k"], case["v"], case["kw"]

    def pin(t):  # a pinned host copy, made without a pageable intermediate
        h = torch.empty(tuple(t.shape), dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h
    if not kv_sharded:
        qh, kh, vh = (pin(x).numpy().view(np.uint16) for x in (q, k, v))
        oh = torch.empty(tuple(out_dev.shape), dtype=torch.int16).pin_memory().numpy().view(np.uint16)
        fh = torch.empty(out_dev.shape[0], dtype=torch.uint8).pin_memory().numpy()
        if name == "c3":
            pt, sl = pin(kw["page_table"]).numpy(), pin(kw["seq_lens"]).numpy()
            h2d = qh.nbytes + kh.nbytes + vh.nbytes + pt.nbytes + sl.nbytes

            def call():
                cuda.attention_cuda_paged(qh, kh, vh, cfg.alpha, pt, sl, kw["q_heads"], splits=splits, out_buf=oh,
                                          flags_buf=fh)
            path = "ea_attention_cuda_paged (host pointers, pinned)"
        else:
            kb, kl = pin(kw["kv_base"]).numpy(), pin(kw["kv_len"]).numpy()
            h2d = qh.nbytes + kh.nbytes + vh.nbytes + kb.nbytes + kl.nbytes

            def call():
                cuda.attention_cuda_ranges(qh, kh, vh, cfg.alpha, kb, kl, kw["max_row_keys"], splits=splits,
                                           out_buf=oh, flags_buf=fh)
            path = "ea_attention_cuda_ranges (host pointers, pinned)"
        d2h = oh.nbytes + fh.nbytes
    else:
        from exactattention_b200 import dist as ea_dist

        host = {n: pin(t) for n, t in (("q", q), ("k", k), ("v", v), ("kv_base", kw["kv_base"]),
                                       ("kv_len", kw["kv_len"]), ("segments", kw["segments"]))}
        dev = {n: torch.empty_like(t, device=R.dev) for n, t in host.items()}
        oh = torch.empty(tuple(out_dev.shape), dtype=torch.int16).pin_memory()
        fh = torch.empty(out_dev.shape[0], dtype=torch.uint8).pin_memory()
        parts = cuda.Partials(q.shape[0], 128, R.dev)
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        d2h = oh.numel() * 2 + fh.numel()

        def call():
            for n_, t in host.items():
                dev[n_].copy_(t, non_blocking=True)
            o, f = ea_dist.attention_kv_sharded(dev["q"], dev["k"], dev["v"], cfg.alpha,
                                                max_row_keys=kw["max_row_keys"], splits=splits, parts=parts,
                                                kv_base=dev["kv_base"], kv_len=dev["kv_len"],
                                                segments=dev["segments"], segment_width=kw.get("segment_width", 0))
            oh.copy_(o, non_blocking=True)
            fh.copy_(f, non_blocking=True)
            torch.cuda.current_stream(R.dev).synchronize()
        path = "dist.attention_kv_sharded (each rank's key shard H2D from pinned host, outputs D2H)"
    for _ in range(2):
        call()
    R.barrier()
    t0 = time.perf_counter()
    steps = 3
    for _ in range(steps):
        call()
    e_ms = R.max((time.perf_counter() - t0) * 1000 / steps)
    o_host = oh if isinstance(oh, np.ndarray) else oh.numpy().view(np.uint16)
    same = bool(np.array_equal(o_host, out_dev.cpu().numpy().view(np.uint16)))
    return {"value": job_pairs / (e_ms / 1000.0), "unit": "pairs/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": e_ms, "steps": steps, "matches_device_output": same,
            "path": path, "h2d_bytes_per_step_is": "per rank" if kv_sharded else "whole job"}


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch

    from exactattention_b200 import build

    R = Runner()
    build.build()
    name = args.config
    head = run_config(R, name, args, headline=True)
    extras = {}
    if args.extras != "none" and not args.kv_shard and not args.seqs:
        for x in [s for s in args.extras.split(",") if s and s != name]:
            extras[x] = run_config(R, x, args, headline=False)
    clk = head.pop("clocks")
    for x in extras.values():
        x.pop("clocks", None)
    R.barrier()
    if R.world > 1:
        R.dist.destroy_process_group()
    if R.rank != 0:
        return

    cpu = None
    if not args.no_cpu and R.world == 1 and not args.kv_shard and not args.seqs:
        from oracle import ref

        if ref.available():
            cores = os.cpu_count() or 1
            cpu_reference_step(name, cores)  # warm-up (page-in, thread start)
            p_, s_, n_, th, fl = cpu_reference_step(name, cores)
            cpu = {"value": p_ / s_, "unit": "pairs/s", "cores": th, "kind": "reference",
                   "sample": cpu_sample_desc(name, n_, th, p_, s_, fl)}
    e2e_rec = head.pop("e2e", None)
    steps_all = args.steps
    line = {
        "metric": "certified QK pairs/s", "value": head["value"], "unit": "pairs/s", "n_gpus": R.world,
        "steps": steps_all, "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "decode_tokens_per_s": head["decode_tokens_per_s"],
        "config": {"workload": name + (f" key range {args.kv_shard}" if args.kv_shard else "") + (
                       f" first {args.seqs} sequences" if args.seqs else ""),
                   "job_pairs": head["job_pairs"], "rows": head["rows"],
                   "splits": head["splits"], "heads": "16q/8kv", "head_dim": 128, "keys_per_sequence": 1 << 20,
                   "l2": "flushed (256 MiB write) between steps", "parallelism": head["parallelism"],
                   "tokens_per_s": head["decode_tokens_per_s"]},
        "roofline": head["roofline"],
        "cpu_baseline": cpu,
        "e2e": e2e_rec,
        "gpu_launches": args.steps * head["launches_per_step"],
        "clocks": clk,
        "certified": dict(head["certified_per_step"], flags_all_zero=head["flags_all_zero"],
                          sha256=head["sha256"], sha_ok=head["sha_ok"]),
        "extra": {"configs": extras},
    }
    print(json.dumps(line))
    del torch


if __name__ == "__main__":
    main()
