"""KV-range sharding on the GPU: partials of disjoint key ranges, merged max-then-sum, must give
the bits of one launch over the whole range and of the oracle (B200 only).

Ranks are emulated on one GPU (one partials call per key range, the collectives replaced by
torch max / sum over the ranges); the NCCL form runs in test_gpu_multi.py when the box has two
or more GPUs.
"""

import numpy as np
import pytest

from gen import bf16

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)


def merge_local(parts_list):
    """The merge of exactattention_b200.dist.merge_partials over in-process ranges."""
    import torch

    from exactattention_b200 import cuda

    mx = torch.stack([p.i32 for p in parts_list]).max(0).values
    rows, dv = parts_list[0].rows, parts_list[0].dv
    for p in parts_list:
        cuda.rescale_partials(p, mx[:rows], mx[2 * rows:].view(rows, dv))
    out = parts_list[0]
    out.status.copy_(mx[rows:2 * rows])
    for p in parts_list[1:]:
        out.i64 += p.i64
    return out


def finish_local(shard_args, out, flags, max_row_keys, stats=None):
    """The sharded wide tier (exactattention_b200.dist.wide_tier) over in-process ranges, for the
    rows the merged tier-1 partials left at flag 1. shard_args: per range (q, k, v, alpha, mask)."""
    import torch

    from exactattention_b200 import cuda

    need = flags == 1
    if not int(need.sum().item()):
        return 0
    rows = need.nonzero().flatten().to(torch.int32)
    ws = [cuda.wide_partials(q, k, v, a, rows, max_row_keys=max_row_keys, stats=stats, **m)
          for (q, k, v, a, m) in shard_args]
    gmax = torch.stack([w.maxv for w in ws]).max(0).values
    for w in ws:
        cuda.rescale_wide_partials(w, gmax)
    for w in ws[1:]:
        ws[0].sumv += w.sumv
    cuda.finalize_wide_partials(ws[0], gmax, rows, out, flags, stats=stats)
    return rows.numel()


def _bounds(n, shards):
    return [(n * s // shards, n * (s + 1) // shards) for s in range(shards)]


@pytest.mark.parametrize("kind,vkind,d", [("normal", "normal", 128), ("outlier", "wide", 128), ("wide", "normal", 64),
                                          ("dupes", "dupes", 128)])
@pytest.mark.parametrize("shards", [2, 3, 8])
def test_kv_shards_simt_match_full_and_oracle(kind, vkind, d, shards):
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(hash((kind, vkind, d, shards)) & 0xFFFF)
    rows, n = 12, 1500
    Q, K, V = bf16(rng, (rows, d), kind), bf16(rng, (n, d), kind), bf16(rng, (n, d), vkind)
    dev = torch.device("cuda")
    alpha = ea.default_alpha(d)
    kb = np.zeros(rows, np.int64)
    kl = np.full(rows, n, np.int64)
    kl[3] = 0
    kl[5] = 700  # rows whose range ends inside a shard or before it: empty partials there
    full, fflags = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev))
    parts, shard_args = [], []
    for i, (lo, hi) in enumerate(_bounds(n, shards)):
        klen = np.clip(kl - lo, 0, hi - lo).astype(np.int64)
        m = dict(kv_base=_t(kb, dev), kv_len=_t(klen, dev))
        shard_args.append((_t(Q, dev), _t(K[lo:hi], dev), _t(V[lo:hi], dev), alpha, m))
        parts.append(cuda.partials(*shard_args[-1][:4], max_row_keys=n, splits=1 + i % 3, **m))
    merged = merge_local(parts)
    out, flags = cuda.finalize_partials(merged, n)
    finish_local(shard_args, out, flags, n)
    torch.cuda.synchronize()
    assert not flags.any().item() and not fflags.any().item()
    assert torch.equal(out, full)
    o = out.cpu().numpy().view(np.uint16)
    for r in (0, 3, 5, rows - 1):
        L = int(kl[r])
        assert np.array_equal(o[r], exact.attention_row(Q[r], K[:L], V[:L], alpha)), r


@pytest.mark.parametrize("shards", [2, 4])
def test_kv_shards_tensor_core_match_full(shards):
    """Causal rows through the tensor-core kernel's export: every shard's rows still form blocks
    sharing a key range."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    rng = np.random.default_rng(40 + shards)
    S, heads = 640, 2
    Q = bf16(rng, (heads * S, 128), "outlier")
    K, V = bf16(rng, (S, 128), "outlier"), bf16(rng, (S, 128), "wide")
    kb = np.zeros(heads * S, np.int64)
    kl = np.tile(np.arange(1, S + 1, dtype=np.int64), heads)
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    full, fflags = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev),
                               blocks=_t(cuda.row_blocks(kb, kl), dev))
    parts, shard_args = [], []
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    for lo, hi in _bounds(S, shards):
        klen = np.clip(kl - lo, 0, hi - lo).astype(np.int64)
        m = dict(kv_base=_t(kb, dev), kv_len=_t(klen, dev))
        shard_args.append((_t(Q, dev), _t(K[lo:hi], dev), _t(V[lo:hi], dev), alpha, m))
        parts.append(cuda.partials(*shard_args[-1][:4], max_row_keys=S, blocks=_t(cuda.row_blocks(kb, klen), dev),
                                   stats=st, **m))
    out, flags = cuda.finalize_partials(merge_local(parts), S)
    finish_local(shard_args, out, flags, S)
    torch.cuda.synchronize()
    assert st.cpu().numpy()[7] == int(kl.sum()), "the tensor-core kernel did not run"
    assert not flags.any().item() and not fflags.any().item()
    assert torch.equal(out, full)


def test_kv_shards_domain_error_propagates():
    """A NaN key in one shard makes the merged row a domain error (flag 2, zero output)."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    rng = np.random.default_rng(9)
    rows, n, d = 6, 400, 64
    Q, K, V = bf16(rng, (rows, d)), bf16(rng, (n, d)), bf16(rng, (n, d))
    K[350, 3] = 0x7F80
    dev = torch.device("cuda")
    alpha = ea.default_alpha(d)
    kb = np.zeros(rows, np.int64)
    kl = np.array([n, 300, n, 351, 350, n], np.int64)
    full, fflags = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev))
    parts, shard_args = [], []
    for lo, hi in _bounds(n, 2):
        klen = np.clip(kl - lo, 0, hi - lo).astype(np.int64)
        m = dict(kv_base=_t(kb, dev), kv_len=_t(klen, dev))
        shard_args.append((_t(Q, dev), _t(K[lo:hi], dev), _t(V[lo:hi], dev), alpha, m))
        parts.append(cuda.partials(*shard_args[-1][:4], max_row_keys=n, **m))
    out, flags = cuda.finalize_partials(merge_local(parts), n)
    finish_local(shard_args, out, flags, n)
    torch.cuda.synchronize()
    assert flags.cpu().numpy().tolist() == [2, 0, 2, 2, 0, 2]
    assert torch.equal(flags, fflags) and torch.equal(out, full)


def test_kv_shards_wide_tier_rows():
    """Rows that only the wide tier certifies merge across shards to the single-launch bits: with
    equal weights, +2^125 (key 0, shard 0) and -2^125 (key 500, shard 1) cancel exactly in
    channel 0, so the int64 windows anchored at 2^125 keep nothing of the result."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(123)
    rows, n, d = 8, 900, 64
    Q = np.zeros((rows, d), np.uint16)          # zero scores: every weight is 1
    K = bf16(rng, (n, d))
    V = bf16(rng, (n, d))
    V[0, 0] = 0x7E00                            # 2^125
    V[500, 0] = 0xFE00                          # -2^125
    dev = torch.device("cuda")
    alpha = ea.default_alpha(d)
    kb = np.zeros(rows, np.int64)
    kl = np.full(rows, n, np.int64)
    st_full = torch.zeros(12, dtype=torch.int64, device=dev)
    full, fflags = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev),
                               stats=st_full)
    parts, shard_args = [], []
    for lo, hi in _bounds(n, 3):
        klen = np.clip(kl - lo, 0, hi - lo).astype(np.int64)
        m = dict(kv_base=_t(kb, dev), kv_len=_t(klen, dev))
        shard_args.append((_t(Q, dev), _t(K[lo:hi], dev), _t(V[lo:hi], dev), alpha, m))
        parts.append(cuda.partials(*shard_args[-1][:4], max_row_keys=n, **m))
    out, flags = cuda.finalize_partials(merge_local(parts), n)
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    n3 = finish_local(shard_args, out, flags, n, stats=st)
    torch.cuda.synchronize()
    assert st_full.cpu().numpy()[2] > 0, "the single launch should need the wide tier here"
    assert n3 > 0
    assert not flags.any().item() and not fflags.any().item()
    assert st.cpu().numpy()[4] == 0
    assert torch.equal(out, full)
    o = out.cpu().numpy().view(np.uint16)
    assert np.array_equal(o[0], exact.attention_row(Q[0], K, V, alpha))


def test_spread_across_shards_is_a_domain_error():
    """Each shard's logits span little, but one shard's lie 2^21 below the other's: the merged row
    breaks the reference's exponent-spread rule (reference.py:30, 116-118) and must be flagged."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda
    from oracle import exact

    f2b = lambda x: np.uint16(exact.f32_to_bits(np.float32(x)) >> 16)  # noqa: E731
    rng = np.random.default_rng(91)
    n, rows = 400, 4
    K, V = bf16(rng, (n, 128)), bf16(rng, (n, 128))
    Q = bf16(rng, (rows, 128))
    Q[:, 0] = f2b(64.0)
    K[:, 0] = 0
    K[200:, 0] = f2b(-262144.0)  # every key of the second half: t ~ -2^21
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    kl = np.array([150, 400, 300, 199], np.int64)
    sees = (kl > 200)
    parts, shard_args = [], []
    for lo, hi in [(0, 200), (200, n)]:
        m = dict(kv_base=t(np.zeros(rows, np.int64)), kv_len=t(np.clip(kl - lo, 0, hi - lo)))
        shard_args.append((t(Q), t(K[lo:hi]), t(V[lo:hi]), alpha, m))
        parts.append(cuda.partials(*shard_args[-1][:4], max_row_keys=n, **m))
    out, flags = cuda.finalize_partials(merge_local(parts), n)
    finish_local(shard_args, out, flags, n)
    torch.cuda.synchronize()
    assert np.array_equal(flags.cpu().numpy() == 2, sees)


def gathered_local(parts_list):
    """The flat buffers of in-process ranges, concatenated (what the all-gather gives every rank)."""
    import torch

    return torch.cat([p.flat for p in parts_list])


@pytest.mark.parametrize("kind,vkind,shards,decode", [("normal", "normal", 3, False), ("outlier", "wide", 8, False),
                                                      ("normal", "heavy", 4, True)])
def test_gathered_merge_equals_two_collective_merge(kind, vkind, shards, decode):
    """The one-collective merge (gather the flat partials, merge and round in one kernel) gives the
    same bits and flags as MAX / rescale / SUM / finalize, and as one launch over all keys; the wide
    rows it lists are exactly the ones the older form flags."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    rng = np.random.default_rng(hash((kind, vkind, shards)) & 0xFFFF)
    rows, n = (4, 4000) if decode else (12, 1500)
    Q, K, V = bf16(rng, (rows, 128), kind), bf16(rng, (n, 128), kind), bf16(rng, (n, 128), vkind)
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    kb = np.zeros(rows, np.int64)
    kl = np.full(rows, n, np.int64)
    if not decode:
        kl[3], kl[5] = 0, 700
    full, fflags = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev))
    parts, parts2, shard_args = [], [], []
    for lo, hi in _bounds(n, shards):
        klen = np.clip(kl - lo, 0, hi - lo).astype(np.int64)
        m = dict(kv_base=_t(kb, dev), kv_len=_t(klen, dev))
        if decode:
            m.update(segments=_t(cuda.row_segments(kb), dev), segment_width=rows, splits=3)
        shard_args.append((_t(Q, dev), _t(K[lo:hi], dev), _t(V[lo:hi], dev), alpha,
                           {k_: v_ for k_, v_ in m.items() if k_ in ("kv_base", "kv_len")}))
        parts.append(cuda.partials(*shard_args[-1][:4], max_row_keys=n, **m))
        parts2.append(cuda.partials(*shard_args[-1][:4], max_row_keys=n, **m))
    out_g, fl_g, wrows, wcount = cuda.merge_gathered(gathered_local(parts), shards, parts[0], n)
    torch.cuda.synchronize()
    out_m, fl_m = cuda.finalize_partials(merge_local(parts2), n)
    torch.cuda.synchronize()
    assert torch.equal(fl_g, fl_m)
    wl = wrows.cpu().numpy()
    nw = int(wcount.item())
    # the wide tier pairs the ranks' partials slot by slot: the list is in row order, then -1
    assert wl[:nw].tolist() == torch.nonzero(fl_m == 1).flatten().cpu().numpy().tolist()
    assert (wl[nw:] == -1).all()
    ok = fl_g == 0
    assert torch.equal(out_g[ok], out_m[ok])
    finish_local(shard_args, out_g, fl_g, n)
    torch.cuda.synchronize()
    assert not fl_g.any().item() and not fflags.any().item()
    assert torch.equal(out_g, full)
