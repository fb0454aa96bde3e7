"""The tensor-core decode kernel (keys on the MMA's M side, a GQA group's rows in N) against the
CUDA-core path and the oracle (B200 only). Every comparison is bit-exact."""

import numpy as np
import pytest

from gen import KINDS, bf16

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)


def _range_case(rng, kind, vkind, nseg, group, L):
    """nseg segments of `group` rows, each segment its own key range; row lengths ragged within a
    segment (the segment reads up to its longest row)."""
    n = nseg * L
    K, V = bf16(rng, (n, 128), kind), bf16(rng, (n, 128), vkind)
    Q = bf16(rng, (nseg * group, 128), kind)
    kb = np.repeat(np.arange(nseg, dtype=np.int64) * L, group)
    kl = rng.integers(1, L + 1, size=nseg * group).astype(np.int64)
    kl[::group] = L
    return Q, K, V, kb, kl


@pytest.mark.parametrize("kind,vkind", [(k, "normal") for k in KINDS] + [("outlier", "wide"), ("dupes", "dupes"),
                                                                         ("heavy", "heavy")])
@pytest.mark.parametrize("group,splits", [(2, 1), (2, 3), (1, 2), (5, 1), (8, 4)])
def test_decode_range_matches_simt_and_oracle(kind, vkind, group, splits):
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(hash((kind, vkind, group, splits)) & 0xFFFF)
    nseg, L = 3, 700
    Q, K, V, kb, kl = _range_case(rng, kind, vkind, nseg, group, L)
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    o_d, f_d = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev),
                           splits=splits, stats=st, segments=_t(cuda.row_segments(kb), dev))
    o_s, f_s = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev))
    torch.cuda.synchronize()
    s = st.cpu().numpy()
    assert s[7] == int(kl.sum()), "the tensor-core decode kernel did not run"
    assert s[5] == int(kl.sum())
    assert torch.equal(f_d, f_s)
    assert torch.equal(o_d, o_s)
    out = o_d.cpu().numpy().view(np.uint16)
    for r in (0, group - 1, len(kl) - 1):
        if f_d[r].item():
            continue
        lo, L_ = int(kb[r]), int(kl[r])
        assert np.array_equal(out[r], exact.attention_row(Q[r], K[lo:lo + L_], V[lo:lo + L_], alpha)), r


def _paged_case(rng, B, hq, hkv, ps, lo, hi, kind="outlier"):
    ctx = rng.integers(lo, hi + 1, size=B)
    npg = (ctx + ps - 1) // ps
    perm = rng.permutation(int(npg.sum())).astype(np.int32)
    maxp = int(npg.max())
    pt = np.zeros((B, maxp), np.int32)
    off = 0
    for b in range(B):
        pt[b, :npg[b]] = perm[off:off + npg[b]]
        off += int(npg[b])
    Kc = bf16(rng, (int(npg.sum()), hkv, ps, 128), kind)
    Vc = bf16(rng, (int(npg.sum()), hkv, ps, 128))
    Q = bf16(rng, (B * hq, 128), kind)
    return Q, Kc, Vc, pt, ctx


@pytest.mark.parametrize("hq,hkv,ps,splits", [(4, 2, 16, 1), (4, 2, 16, 4), (8, 1, 5, 2), (3, 3, 32, 1), (8, 2, 16, 3),
                                             (12, 4, 8, 1)])
def test_decode_paged_matches_csr_and_oracle(hq, hkv, ps, splits):
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(1000 + hq * 10 + ps)
    B = 3
    Q, Kc, Vc, pt, ctx = _paged_case(rng, B, hq, hkv, ps, 1, 600)
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    o_p, f_p = cuda.launch(_t(Q, dev), _t(Kc, dev), _t(Vc, dev), alpha, page_table=_t(pt, dev),
                           seq_lens=_t(ctx.astype(np.int32), dev), page_size=ps, q_heads=hq, kv_heads=hkv,
                           splits=splits, stats=st)
    rows = []
    for r in range(B * hq):
        b, h = divmod(r, hq)
        j = np.arange(ctx[b])
        rows.append((pt[b, j // ps].astype(np.int64) * hkv + h // (hq // hkv)) * ps + j % ps)
    rp = np.concatenate([[0], np.cumsum([len(x) for x in rows])]).astype(np.int64)
    ki = np.concatenate(rows)
    o_c, f_c = cuda.launch(_t(Q, dev), _t(Kc, dev), _t(Vc, dev), alpha, row_ptr=_t(rp, dev), key_idx=_t(ki, dev))
    torch.cuda.synchronize()
    assert st.cpu().numpy()[7] == int(ctx.sum()) * hq, "the tensor-core decode kernel did not run"
    assert not f_p.any().item() and torch.equal(f_p, f_c)
    assert torch.equal(o_p, o_c)
    Kf, Vf = Kc.reshape(-1, 128), Vc.reshape(-1, 128)
    out = o_p.cpu().numpy().view(np.uint16)
    for r in (0, B * hq - 1):
        assert np.array_equal(out[r], exact.attention_row(Q[r], Kf[rows[r]], Vf[rows[r]], alpha)), r


def test_decode_nan_and_empty_rows():
    """A NaN value seen by some rows only; a row with no keys; a padded segment slot."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    rng = np.random.default_rng(4242)
    L = 400
    K, V = bf16(rng, (2 * L, 128)), bf16(rng, (2 * L, 128))
    Q = bf16(rng, (5, 128))
    V[300, 17] = 0x7FC0
    V[299, 17] = 0x4280  # 64.0 next to it: the channel's range must come from the finite values
    kb = np.array([0, 0, 0, L, L], np.int64)
    kl = np.array([L, 300, 0, L, 250], np.int64)
    seg = np.full((3, 8), -1, np.int32)
    seg[0, :2] = [0, 1]
    seg[1, 3] = 2       # padding before a row
    seg[2, :2] = [3, 4]
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    o_d, f_d = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev),
                           segments=_t(seg, dev), splits=2)
    o_s, f_s = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev))
    torch.cuda.synchronize()
    assert f_d.cpu().numpy().tolist() == [2, 0, 0, 0, 0]
    assert torch.equal(f_d, f_s) and torch.equal(o_d, o_s)
    assert not o_d[2].any().item()


def test_decode_kv_sharded_partials():
    """Partials of the decode kernel over key ranges merge to the one-launch bits."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda
    from test_gpu_kv_shard import finish_local, merge_local

    rng = np.random.default_rng(77)
    group, n = 2, 3000
    Q = bf16(rng, (2 * group, 128), "outlier")
    K, V = bf16(rng, (2 * n, 128), "outlier"), bf16(rng, (2 * n, 128), "wide")
    kb_full = np.repeat(np.array([0, n], np.int64), group)
    kl_full = np.full(2 * group, n, np.int64)
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    full, fflags = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, kv_base=_t(kb_full, dev),
                               kv_len=_t(kl_full, dev))
    parts, shard_args = [], []
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    for lo, hi in [(0, 1000), (1000, 1900), (1900, n)]:
        Ks = np.concatenate([K[lo:hi], K[n + lo:n + hi]])
        Vs = np.concatenate([V[lo:hi], V[n + lo:n + hi]])
        kb = np.repeat(np.array([0, hi - lo], np.int64), group)
        kl = np.full(2 * group, hi - lo, np.int64)
        m = dict(kv_base=_t(kb, dev), kv_len=_t(kl, dev))
        shard_args.append((_t(Q, dev), _t(Ks, dev), _t(Vs, dev), alpha, m))
        parts.append(cuda.partials(*shard_args[-1][:4], max_row_keys=n, splits=2, stats=st,
                                   segments=_t(cuda.row_segments(kb), dev), **m))
    out, flags = cuda.finalize_partials(merge_local(parts), n)
    finish_local(shard_args, out, flags, n)
    torch.cuda.synchronize()
    assert st.cpu().numpy()[7] == int(kl_full.sum())
    assert torch.equal(flags, fflags) and torch.equal(out, full)


def test_host_entries_take_the_decode_kernel():
    """Host-pointer entries: ea_attention_cuda_paged (paged caches) and ea_attention_cuda_ranges
    (rows in groups of at most 8 per key range: decode segments built by the library) give the
    device launch's bits."""
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    rng = np.random.default_rng(606)
    B, hq, hkv, ps = 3, 4, 2, 16
    Q, Kc, Vc, pt, ctx = _paged_case(rng, B, hq, hkv, ps, 100, 900)
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    o_d, f_d = cuda.launch(_t(Q, dev), _t(Kc, dev), _t(Vc, dev), alpha, page_table=_t(pt, dev),
                           seq_lens=_t(ctx.astype(np.int32), dev), page_size=ps, q_heads=hq, kv_heads=hkv, splits=3)
    o_h, f_h = cuda.attention_cuda_paged(Q, Kc, Vc, alpha, pt, ctx.astype(np.int32), hq, splits=3)
    assert np.array_equal(o_h, o_d.cpu().numpy().view(np.uint16)) and np.array_equal(f_h, f_d.cpu().numpy())

    Q2, K2, V2, kb, kl = _range_case(rng, "outlier", "normal", 4, 2, 500)
    o_d2, f_d2 = cuda.launch(_t(Q2, dev), _t(K2, dev), _t(V2, dev), alpha, kv_base=_t(kb, dev), kv_len=_t(kl, dev),
                             splits=2)
    cuda.kernel_timing(1)
    o_h2, f_h2 = cuda.attention_cuda_ranges(Q2, K2, V2, alpha, kb, kl, splits=2)
    ms, n = cuda.kernel_timing(2)
    cuda.kernel_timing(0)
    assert n == 1 and ms > 0
    assert np.array_equal(o_h2, o_d2.cpu().numpy().view(np.uint16)) and np.array_equal(f_h2, f_d2.cpu().numpy())
