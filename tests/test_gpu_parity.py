"""Parity of the CUDA path with the oracle and the reference's golden vectors (B200 only).

Every comparison is bit-exact: the spec defines one correct output per input.
"""

import hashlib
import json
import os

import numpy as np
import pytest

from gen import KINDS, bf16

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def ea(cuda_lib):
    import torch

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    import exactattention_b200 as ea

    return ea


# ---------------------------------------------------------------------------
# golden vectors of the reference
# ---------------------------------------------------------------------------

def test_config1_golden(ea):
    z = np.load(os.path.join(GOLDEN, "c1.npz"))
    out = ea.attention(z["q"], z["k"], z["v"], z["alpha"])
    assert sha(out) == "27b27a491d2064580a707b042c162d42e3a5f2ca4232043d3de870c840922843"
    assert np.array_equal(out, z["out"])
    out32 = ea.attention(z["q"], z["k"], z["v"], z["alpha"], out="fp32")
    assert np.array_equal(out32.view(np.uint32), z["out32"].view(np.uint32))


def test_small_cases_golden(ea):
    z = np.load(os.path.join(GOLDEN, "small_cases.npz"))
    for i in range(int(z["count"])):
        key = f"case{i}"
        fmt = str(z[key + "_fmt"])
        out = ea.attention(z[key + "_q"], z[key + "_k"], z[key + "_v"], z[key + "_alpha"], mask=z[key + "_mask"],
                           out=fmt)
        exp = z[key + "_out"]
        if fmt == "fp32":
            assert np.array_equal(out.view(np.uint32), exp.view(np.uint32)), key
        else:
            assert np.array_equal(out, exp), key


@pytest.mark.parametrize("splits", [1, 8])
def test_fixture_heads_sha(ea, splits):
    """The reference's portable fixture (scripts/fixture.py check): every causal row of two
    real Qwen3-0.6B heads hashes to the recorded SHA-256."""
    from exactattention_b200.cuda import CudaStats, attention_cuda

    z = np.load(os.path.join(GOLDEN, "qwen3_heads.npz"))
    exp = json.load(open(os.path.join(GOLDEN, "qwen3_heads.json")))
    for key, info in exp["heads"].items():
        q, k, v, a = z["q_" + key], z["k_" + key], z["v_" + key], np.float32(z["alpha_" + key])
        L = q.shape[0]
        kv = np.arange(1, L + 1)
        rp = np.concatenate([[0], np.cumsum(kv)]).astype(np.int64)
        ki = np.concatenate([np.arange(n) for n in kv]).astype(np.int64)
        st = CudaStats()
        out, flags = attention_cuda(q, k, v, a, rp, ki, splits=splits, stats=st)
        assert sha(out) == info["sha256"], key
        assert not flags.any() and st.host_fallbacks == 0
        from exactattention_b200 import _lib

        full = _lib.last_host_stats()
        assert full["tc_pairs"] == full["pairs"] == int(kv.sum()), full  # every pair on the tensor cores


def _csr(rows_keys):
    rp = np.concatenate([[0], np.cumsum([len(x) for x in rows_keys])]).astype(np.int64)
    ki = np.concatenate(rows_keys).astype(np.int64)
    return rp, ki


def test_csr_entry_reaches_tensor_cores(ea):
    """The reference's C entry with CSR lists (ea_attention_cuda): causal rows run on the
    tensor-core prefill kernel, tree rows (prefix + ancestors) on it plus the CUDA-core list
    kernel, a GQA decode group on the decode kernel. Bits equal the CUDA-core CSR path and the
    oracle."""
    import torch

    from exactattention_b200 import _lib, cuda
    from exactattention_b200.cuda import attention_cuda
    from oracle import exact

    rng = np.random.default_rng(21)
    alpha = ea.default_alpha(128)
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    cases = []
    S = 300  # causal prefill, two heads
    cases.append(("causal", bf16(rng, (2 * S, 128), "outlier"), bf16(rng, (S, 128), "outlier"),
                  bf16(rng, (S, 128)), [np.arange(r % S + 1) for r in range(2 * S)], 2 * (S * (S + 1) // 2)))
    P, T = 500, 40  # tree verification: prefix + ancestors, node keys after the prefix
    parent = [-1] + [int(rng.integers(0, i)) for i in range(1, T)]
    tree_rows = []
    for h in range(2):
        for i in range(T):
            path, x = [], i
            while x != -1:
                path.append(P + x)
                x = parent[x]
            tree_rows.append(np.concatenate([np.arange(P), np.sort(np.array(path))]))
    cases.append(("tree", bf16(rng, (2 * T, 128)), bf16(rng, (P + T, 128), "outlier"), bf16(rng, (P + T, 128)),
                  tree_rows, None))
    n = 700  # one GQA decode group
    cases.append(("decode", bf16(rng, (2, 128)), bf16(rng, (n, 128), "heavy"), bf16(rng, (n, 128)),
                  [np.arange(n), np.arange(n)], 2 * n))
    for name, Q, K, V, rows_keys, tc_pairs in cases:
        rp, ki = _csr(rows_keys)
        out, flags = attention_cuda(Q, K, V, alpha, rp, ki, splits=8)
        st = _lib.last_host_stats()
        assert not flags.any()
        if tc_pairs is not None:
            assert st["tc_pairs"] == tc_pairs == st["pairs"], (name, st)
        else:
            assert st["tc_pairs"] >= 2 * T * (P - 64), (name, st)  # the prefix part
        o_s, _ = cuda.launch(t(Q), t(K), t(V), alpha, row_ptr=t(rp), key_idx=t(ki))  # CUDA-core CSR kernel
        assert np.array_equal(out, o_s.cpu().numpy().view(np.uint16)), name
        for r in (0, len(rows_keys) // 2, len(rows_keys) - 1):
            sel = rows_keys[r]
            assert np.array_equal(out[r], exact.attention_row(Q[r], K[sel], V[sel], alpha)), (name, r)


@pytest.mark.parametrize("splits", [1, 2, 5, 16])
def test_tensor_core_prefill_kv_splits(ea, splits):
    """The prefill kernel's KV splits (grid y, tile-aligned key ranges, exact split combine) give
    the same bits at every split count, all pairs on the tensor cores."""
    import torch

    from exactattention_b200 import cuda

    rng = np.random.default_rng(31)
    S = 700
    Q = bf16(rng, (2 * S, 128), "outlier")
    K, V = bf16(rng, (S, 128), "outlier"), bf16(rng, (S, 128), "wide")
    kb = np.zeros(2 * S, np.int64)
    kl = np.tile(np.arange(1, S + 1, dtype=np.int64), 2)
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    st = cuda.new_stats(dev)
    o, f = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), splits=splits, stats=st,
                       blocks=t(cuda.row_blocks(kb, kl)))
    o_s, f_s = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl))
    torch.cuda.synchronize()
    assert not f.any().item()
    assert st.cpu().numpy()[7] == int(kl.sum())
    assert torch.equal(o, o_s)


# ---------------------------------------------------------------------------
# random inputs vs the exact oracle
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("out", ["bf16", "fp32"])
def test_random_rows_match_oracle(ea, kind, out):
    from oracle import exact

    from exactattention_b200.cuda import attention_cuda

    rng = np.random.default_rng(hash((kind, out)) & 0xFFFF)
    for trial in range(3):
        d = int(rng.choice([16, 64, 128]))
        dv = int(rng.choice([8, 32, 64, 128]))
        n = int(rng.integers(1, 300))
        vkind = ["normal", "wide", "dupes"][trial]
        Q, K, V = bf16(rng, (3, d), kind), bf16(rng, (n, d), kind), bf16(rng, (n, dv), vkind)
        alpha = exact.default_alpha(d)
        splits = int(rng.integers(1, 9))
        got, flags = attention_cuda(Q, K, V, alpha, out=out, splits=splits)
        exp = exact.attention(Q, K, V, alpha, out=out)
        assert not flags.any()
        if out == "fp32":
            assert np.array_equal(got.view(np.uint32), exp.view(np.uint32)), (kind, trial)
        else:
            assert np.array_equal(got, exp), (kind, trial)


def test_schedule_invariance(ea):
    """Any split count and any key order give the same bits (SPEC 5.3; the reference's
    test_schedule_invariance_many_schedules)."""
    from exactattention_b200.cuda import attention_cuda
    from oracle import exact

    rng = np.random.default_rng(11)
    d, dv, n, r = 128, 64, 700, 8
    Q, K, V = bf16(rng, (r, d), "outlier"), bf16(rng, (n, d), "outlier"), bf16(rng, (n, dv))
    alpha = exact.default_alpha(d)
    base, flags = attention_cuda(Q, K, V, alpha)
    assert not flags.any()
    for splits in (2, 3, 7, 16, 64):
        for perm_seed in (0, 1):
            perm = np.random.default_rng(perm_seed).permutation(n)
            rp = np.arange(r + 1, dtype=np.int64) * n
            ki = np.tile(perm, r).astype(np.int64)
            got, fl = attention_cuda(Q, K, V, alpha, rp, ki, splits=splits)
            assert not fl.any() and np.array_equal(got, base), (splits, perm_seed)
    for i in range(2):
        assert np.array_equal(base[i], exact.attention_row(Q[i], K, V, alpha))


def test_tree_mask_csr_equals_sequential(ea):
    """Each tree node (prefix + ancestors) equals sequential decoding of its root-to-node path."""
    from exactattention_b200.cuda import attention_cuda
    from oracle import exact

    rng = np.random.default_rng(5)
    d, dv, P, T = 64, 32, 300, 15
    parent = [-1] + [int(rng.integers(0, i)) for i in range(1, T)]
    Kp, Vp = bf16(rng, (P, d)), bf16(rng, (P, dv))
    Kt, Vt, Qt = bf16(rng, (T, d)), bf16(rng, (T, dv)), bf16(rng, (T, d))
    K, V = np.concatenate([Kp, Kt]), np.concatenate([Vp, Vt])
    rows = []
    for i in range(T):
        path, x = [], i
        while x != -1:
            path.append(P + x)
            x = parent[x]
        rows.append(np.concatenate([np.arange(P), np.array(path)]))
    rp = np.concatenate([[0], np.cumsum([len(x) for x in rows])]).astype(np.int64)
    ki = np.concatenate(rows).astype(np.int64)
    alpha = exact.default_alpha(d)
    tree, flags = attention_cuda(Qt, K, V, alpha, rp, ki, splits=4)
    assert not flags.any()
    for i in range(T):
        seq_idx = np.sort(rows[i])
        seq, _ = attention_cuda(Qt[i:i + 1], K[seq_idx], V[seq_idx], alpha)
        assert np.array_equal(tree[i], seq[0])
        assert np.array_equal(tree[i], exact.attention_row(Qt[i], K[seq_idx], V[seq_idx], alpha))


def test_nan_inf_rows_flagged(ea):
    """Rows that see a NaN/inf (q, or an attended key/value) get flag 2; the others are exact."""
    import torch

    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(3)
    d, dv, n = 32, 16, 40
    Q, K, V = bf16(rng, (6, d)), bf16(rng, (n, d)), bf16(rng, (n, dv))
    Q[1, 3] = 0x7FC0        # NaN in q row 1
    K[10, 2] = 0x7F80       # +inf in key 10
    V[20, 5] = 0xFF80       # -inf in value 20
    mask = np.ones((6, n), bool)
    mask[2:, 10] = False    # rows 2.. skip key 10
    mask[3:, 20] = False    # rows 3.. skip key 20
    rp, ki = exact.csr_from_mask(mask)
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    out, flags = cuda.launch(t(Q), t(K), t(V), exact.default_alpha(d), row_ptr=t(rp), key_idx=t(ki))
    flags = flags.cpu().numpy()
    assert flags.tolist() == [2, 2, 2, 0, 0, 0]
    out = out.cpu().numpy().view(np.uint16)
    for r in (3, 4, 5):
        sel = np.flatnonzero(mask[r])
        assert np.array_equal(out[r], exact.attention_row(Q[r], K[sel], V[sel], exact.default_alpha(d)))
    with pytest.raises(ea.ExactAttentionDomainError):
        ea.attention(Q, K, V, exact.default_alpha(d), mask=mask)


def test_empty_rows_and_single_key(ea):
    from exactattention_b200.cuda import attention_cuda
    from oracle import exact

    rng = np.random.default_rng(2)
    d, dv = 16, 8
    Q, K, V = bf16(rng, (3, d)), bf16(rng, (5, d)), bf16(rng, (5, dv))
    rp = np.array([0, 0, 1, 1], np.int64)
    ki = np.array([4], np.int64)
    out, flags = attention_cuda(Q, K, V, exact.default_alpha(d), rp, ki)
    assert not flags.any()
    assert np.array_equal(out[0], np.zeros(dv, np.uint16)) and np.array_equal(out[2], np.zeros(dv, np.uint16))
    assert np.array_equal(out[1], V[4])          # one key returns its value exactly


def test_identical_keys_average_values(ea):
    from exactattention_b200.cuda import attention_cuda
    from exactattention_b200.formats import bf16_bits_to_float32
    from oracle import exact

    rng = np.random.default_rng(1)
    q = bf16(rng, (1, 32))
    k = np.repeat(bf16(rng, (1, 32)), 4, axis=0)
    v = bf16(rng, (4, 32))
    out, _ = attention_cuda(q, k, v, exact.default_alpha(32), out="fp32")
    vf = bf16_bits_to_float32(v).astype(np.float64)
    assert np.array_equal(out[0], np.float32(vf.mean(axis=0)))


def test_round_ratio_export(ea):
    """ea_round_ratio_cuda against the reference's round_rational known answers."""
    from exactattention_b200.cuda import round_ratio

    z = np.load(os.path.join(GOLDEN, "round_kat.npz"))
    abEf, val, ovf = z["abEf"], z["val"], z["ovf"]
    for i in range(0, len(val), 7):
        a, b, E, is32 = (int(x) for x in abEf[i])
        got, ov = round_ratio(a, b, E, False, bool(is32))
        if ovf[i]:
            assert ov
        else:
            assert not ov and got == val[i], (a, b, E, is32)


# ---------------------------------------------------------------------------
# device API mask layouts and the synthetic generator
# ---------------------------------------------------------------------------

def test_synth_device_matches_numpy(ea):
    import torch

    from exactattention_b200 import workloads as w

    cfg = w.config("c2")
    dk = w.synth_device(2, w.T_K, (1, 8, 4096, 128), cfg.k_scale).cpu().numpy().view(np.uint16)
    for h in (0, 5):
        assert np.array_equal(dk[0, h, 100:400], w.synth_rows(2, w.T_K, (1, 8, 4096, 128), 0, h, 100, 400, cfg.k_scale))
    sh = w.synth_device(5, w.T_K, (4, 8, 1000, 128), None, 10, t0=5000, T_full=1 << 20).cpu().numpy().view(np.uint16)
    assert np.array_equal(sh[3, 6], w.synth_rows(5, w.T_K, (4, 8, 1 << 20, 128), 3, 6, 5000, 6000, None, 10))
    del torch


def test_layouts_agree(ea):
    """RANGE, PAGED and HYBRID descriptions of the same key sets give the CSR result."""
    import torch

    from exactattention_b200 import cuda

    rng = np.random.default_rng(9)
    dev = torch.device("cuda")
    B, hq, hkv, d, ps = 3, 4, 2, 64, 16
    ctx = rng.integers(1, 200, size=B)
    npg = (ctx + ps - 1) // ps
    perm = rng.permutation(int(npg.sum())).astype(np.int32)
    maxp = int(npg.max())
    pt = np.zeros((B, maxp), np.int32)
    off = 0
    for b in range(B):
        pt[b, :npg[b]] = perm[off:off + npg[b]]
        off += int(npg[b])
    Kc = bf16(rng, (int(npg.sum()), hkv, ps, d), "outlier")
    Vc = bf16(rng, (int(npg.sum()), hkv, ps, d))
    Q = bf16(rng, (B * hq, d), "outlier")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(d)
    o_p, f_p = cuda.launch(t(Q), t(Kc), t(Vc), alpha, page_table=t(pt), seq_lens=t(ctx.astype(np.int32)),
                           page_size=ps, q_heads=hq, kv_heads=hkv, splits=3)
    # the same keys as CSR rows of the flattened cache
    rows = []
    for r in range(B * hq):
        b, h = divmod(r, hq)
        j = np.arange(ctx[b])
        rows.append(((pt[b, j // ps].astype(np.int64) * hkv + h // (hq // hkv)) * ps + j % ps))
    rp = np.concatenate([[0], np.cumsum([len(x) for x in rows])]).astype(np.int64)
    ki = np.concatenate(rows)
    o_c, f_c = cuda.launch(t(Q), t(Kc), t(Vc), alpha, row_ptr=t(rp), key_idx=t(ki))
    assert not f_p.any().item() and not f_c.any().item()
    assert torch.equal(o_p, o_c)
    # HYBRID: first 5 keys as a range over a copied contiguous cache, rest as CSR
    Kf, Vf = Kc.reshape(-1, d), Vc.reshape(-1, d)
    base = np.array([x[0] for x in rows], np.int64)
    contig = [np.arange(len(x)) for x in rows]
    Kl = np.concatenate([Kf[x] for x in rows])
    Vl = np.concatenate([Vf[x] for x in rows])
    starts = np.concatenate([[0], np.cumsum([len(x) for x in rows])[:-1]]).astype(np.int64)
    n0 = np.minimum(5, [len(x) for x in rows]).astype(np.int64)
    tails = [starts[i] + contig[i][n0[i]:] for i in range(len(rows))]
    rp2 = np.concatenate([[0], np.cumsum([len(x) for x in tails])]).astype(np.int64)
    ki2 = np.concatenate(tails).astype(np.int64)
    o_h, f_h = cuda.launch(t(Q), t(Kl), t(Vl), alpha, kv_base=t(starts), kv_len=t(n0), row_ptr=t(rp2),
                           key_idx=t(ki2), splits=2)
    assert torch.equal(o_h, o_c)
    del base


# ---------------------------------------------------------------------------
# full configurations vs the reference's SHA-256
# ---------------------------------------------------------------------------

def _configs():
    p = os.path.join(GOLDEN, "configs.json")
    return json.load(open(p)) if os.path.exists(p) else {}


@pytest.mark.parametrize("name,splits", [("c2", 1), ("c3", 1), ("c3", 4), ("c3", 16), ("c4", 1), ("c5", 4)])
def test_config_sha(ea, name, splits):
    import torch

    from exactattention_b200 import cuda, workloads as w

    gold = _configs()
    if name not in gold:
        pytest.skip(f"no golden SHA for {name}")
    case = w.device_case(name)
    stats = torch.zeros(12, dtype=torch.int64, device="cuda")
    out, flags = cuda.launch(case["q"], case["k"], case["v"], case["cfg"].alpha, splits=splits, stats=stats,
                             **case["kw"])
    torch.cuda.synchronize()
    assert not flags.any().item()
    assert sha(out.cpu().numpy().view(np.uint16)) == gold[name], name
    st = stats.cpu().numpy()
    assert st[6] == 0 and st[4] == 0
    assert st[5] == case["cfg"].pairs


@pytest.mark.parametrize("seqs", [(0, 9)])
def test_config4_tree_equals_sequential_decode(ea, seqs):
    """Config 4 (speculative tree verification): every node row of the listed sequences, computed
    as one tree launch (the 8192-key prefix on the tensor-core prefill kernel, the ancestor lists
    on the CUDA cores, merged), has the bits of one-token decoding along its root-to-node path:
    the tensor-core decode kernel over the prefix and the path's keys gathered into contiguous
    rows (the reference checks the same identity on its CPU kernel, test_cpu_kernel.py:77-104)."""
    import torch

    from exactattention_b200 import cuda, workloads as w

    case = w.device_case("c4")
    cfg, kw = case["cfg"], case["kw"]
    st = torch.zeros(12, dtype=torch.int64, device="cuda")
    tree, flags = cuda.launch(case["q"], case["k"], case["v"], cfg.alpha, splits=3, stats=st, **kw)
    torch.cuda.synchronize()
    assert not flags.any().item()
    assert int(st[7].item()) >= cfg.rows * cfg.prefix  # the prefixes ran on the tensor cores
    P, Tq, T = cfg.prefix, cfg.q_tokens, cfg.kv_tokens
    dev = case["k"].device
    for b in seqs:
        # gathered key rows: (kv head, node) -> prefix + the node's path, at slot (kvh * Tq + x) * (P + 8)
        span = P + 8
        idx, kl = [], []
        for kvh in range(w.HKV):
            base = (b * w.HKV + kvh) * T
            for x in range(Tq):
                path = np.array(cfg.ancestors(b, x), np.int64)
                keys = np.concatenate([np.arange(P), P + path]) + base
                idx.append(np.pad(keys, (0, span - len(keys)), constant_values=base))
                kl.append(len(keys))
        idx = torch.from_numpy(np.concatenate(idx)).to(dev)
        Kg, Vg = case["k"].index_select(0, idx), case["v"].index_select(0, idx)
        rows = np.arange(b * w.HQ * Tq, (b + 1) * w.HQ * Tq)  # canonical order (b, h, node)
        h, x = (rows // Tq) % w.HQ, rows % Tq
        slot = (h // w.GROUP) * Tq + x
        base_g = (slot * span).astype(np.int64)
        len_g = np.array(kl, np.int64)[slot]
        q = case["q"][torch.from_numpy(rows).to(dev)]
        seq, f2 = cuda.launch(q, Kg, Vg, cfg.alpha, kv_base=torch.from_numpy(base_g).to(dev),
                              kv_len=torch.from_numpy(len_g).to(dev), max_row_keys=span,
                              segments=torch.from_numpy(cuda.row_segments(base_g)).to(dev), segment_width=2,
                              splits=4)
        torch.cuda.synchronize()
        assert not f2.any().item()
        assert torch.equal(seq, tree[torch.from_numpy(rows).to(dev)]), f"sequence {b}"


# ---------------------------------------------------------------------------
# tensor-core (tcgen05) prefill kernel
# ---------------------------------------------------------------------------

def _causal_case(rng, S, kind, vkind, heads=2):
    Q = bf16(rng, (heads * S, 128), kind)
    K = bf16(rng, (S, 128), kind)
    V = bf16(rng, (S, 128), vkind)
    kv_base = np.zeros(heads * S, np.int64)
    kv_len = np.tile(np.arange(1, S + 1, dtype=np.int64), heads)
    return Q, K, V, kv_base, kv_len


@pytest.mark.parametrize("kind,vkind", [("normal", "normal"), ("outlier", "wide"), ("wide", "normal"),
                                        ("dupes", "dupes"), ("subnormal", "normal")])
def test_tensor_core_prefill_matches_simt_and_oracle(ea, kind, vkind):
    import torch

    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(hash((kind, vkind)) & 0xFFFF)
    S = 300
    Q, K, V, kb, kl = _causal_case(rng, S, kind, vkind)
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    st_tc = torch.zeros(12, dtype=torch.int64, device=dev)
    o_tc, f_tc = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), stats=st_tc,
                             blocks=t(cuda.row_blocks(kb, kl)))
    o_s, f_s = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl))
    torch.cuda.synchronize()
    st = st_tc.cpu().numpy()
    assert st[7] == int(kl.sum()), "the tensor-core kernel did not run"
    assert torch.equal(f_tc, f_s)
    assert torch.equal(o_tc, o_s)
    out = o_tc.cpu().numpy().view(np.uint16)
    for r in (0, 1, 17, 150, S - 1, S, 2 * S - 1):
        L = int(kl[r])
        assert np.array_equal(out[r], exact.attention_row(Q[r], K[:L], V[:L], alpha)), r


def test_tensor_core_ragged_blocks_and_nan(ea):
    """Blocks with padding rows, rows of different ranges, and a NaN key that only some rows see."""
    import torch

    from exactattention_b200 import cuda

    rng = np.random.default_rng(77)
    n = 500
    K, V = bf16(rng, (n, 128), "outlier"), bf16(rng, (n, 128))
    Q = bf16(rng, (333, 128), "outlier")
    kb = rng.choice([0, 100, 250], size=333).astype(np.int64)
    kl = rng.integers(0, n - 250, size=333).astype(np.int64)
    K[180, 5] = 0x7FC0
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    o_tc, f_tc = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), stats=st,
                             blocks=t(cuda.row_blocks(kb, kl)))
    o_s, f_s = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl))
    torch.cuda.synchronize()
    assert st.cpu().numpy()[7] == int(kl.sum())
    sees = (kb <= 180) & (180 < kb + kl)
    assert np.array_equal(f_tc.cpu().numpy() == 2, sees)
    assert torch.equal(f_tc, f_s)
    ok = torch.from_numpy(~sees).to(dev)
    assert torch.equal(o_tc[ok], o_s[ok])


def test_host_ranges_row_orders_and_threads(ea):
    """ea_attention_cuda_ranges builds the prefill row blocks itself: rows in causal order (one
    pass), rows permuted (sorted), and ragged ranges give the device launch's bits; calls from
    several threads at once (the host entry is reentrant, as the reference's is) give each
    call's sequential result."""
    import threading

    import torch

    from exactattention_b200 import cuda

    rng = np.random.default_rng(515)
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    cases = []
    for S, heads in ((300, 2), (520, 3)):
        Q, K, V, kb, kl = _causal_case(rng, S, "outlier", "normal", heads)
        cases.append((Q, K, V, kb, kl))
    perm = rng.permutation(len(cases[0][0]))
    Q, K, V, kb, kl = cases[0]
    cases.append((Q[perm].copy(), K, V, kb[perm].copy(), kl[perm].copy()))
    n = 700
    K3, V3 = bf16(rng, (n, 128), "outlier"), bf16(rng, (n, 128))
    kb3 = rng.choice([0, 90, 200, 350], size=400).astype(np.int64)
    kl3 = rng.integers(1, n - 350, size=400).astype(np.int64)
    cases.append((bf16(rng, (400, 128), "outlier"), K3, V3, kb3, kl3))
    ref = []
    for Q, K, V, kb, kl in cases:
        o_d, f_d = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl))
        ref.append((o_d.cpu().numpy().view(np.uint16), f_d.cpu().numpy()))
        o_h, f_h = cuda.attention_cuda_ranges(Q, K, V, alpha, kb, kl)
        assert np.array_equal(o_h, ref[-1][0]) and np.array_equal(f_h, ref[-1][1])
    o0 = ref[0][0]
    assert np.array_equal(ref[2][0], o0[perm])
    res = [None] * 12
    errs = []

    def work(i):
        try:
            Q, K, V, kb, kl = cases[i % len(cases)]
            res[i] = cuda.attention_cuda_ranges(Q, K, V, alpha, kb, kl)
        except Exception as e:  # noqa: BLE001 - reported below
            errs.append(repr(e))

    th = [threading.Thread(target=work, args=(i,)) for i in range(len(res))]
    for x in th:
        x.start()
    for x in th:
        x.join()
    assert not errs, errs
    for i, (o, f) in enumerate(res):
        assert np.array_equal(o, ref[i % len(cases)][0]) and np.array_equal(f, ref[i % len(cases)][1]), i


def test_tensor_core_value_channel_edges(ea):
    """Value channels the tensor-core kernel must not take the fast conversion for: all zeros but
    one NaN (seen by some rows only), a subnormal next to normal values (bits below the window),
    an infinity; against the CUDA-core path, flags included."""
    import torch

    from exactattention_b200 import cuda

    rng = np.random.default_rng(78)
    n = 400
    K, V = bf16(rng, (n, 128), "outlier"), bf16(rng, (n, 128))
    Q = bf16(rng, (300, 128), "outlier")
    V[:, 7] = 0
    V[300, 7] = 0x7FC0     # NaN in an otherwise zero channel
    V[40, 9] = 0x0001      # subnormal among normal values
    V[41, 9] = 0x8003
    V[200, 11] = 0xFF80    # -inf
    kb = np.zeros(300, np.int64)
    kl = rng.integers(1, n + 1, size=300).astype(np.int64)
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    o_tc, f_tc = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), stats=st,
                             blocks=t(cuda.row_blocks(kb, kl)))
    o_s, f_s = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl))
    torch.cuda.synchronize()
    assert st.cpu().numpy()[7] == int(kl.sum())
    sees = kl > 200
    assert np.array_equal(f_tc.cpu().numpy() == 2, sees)
    assert torch.equal(f_tc, f_s)
    ok = torch.from_numpy(~sees).to(dev)
    assert torch.equal(o_tc[ok], o_s[ok])


def test_tensor_core_hybrid_tree_mask(ea):
    """HYBRID masks with row blocks: the shared prefix on the tensor cores, the ancestor lists on
    the CUDA cores, merged; equal to the CUDA-core path and to sequential decode (oracle)."""
    import torch

    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(314)
    P, nodes, heads = 500, 24, 2
    parent = [-1] + [int(rng.integers(0, i)) for i in range(1, nodes)]
    K = bf16(rng, (P + nodes, 128), "outlier")
    V = bf16(rng, (P + nodes, 128))
    Q = bf16(rng, (heads * nodes, 128), "outlier")
    anc = []
    for i in range(nodes):
        a, x = [], i
        while x >= 0:
            a.append(x)
            x = parent[x]
        anc.append(sorted(a))
    tails = [np.array(anc[r % nodes], np.int64) + P for r in range(heads * nodes)]
    rp = np.concatenate([[0], np.cumsum([len(x) for x in tails])]).astype(np.int64)
    ki = np.concatenate(tails).astype(np.int64)
    kb = np.zeros(heads * nodes, np.int64)
    kl = np.full(heads * nodes, P, np.int64)
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    o_tc, f_tc = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), row_ptr=t(rp), key_idx=t(ki),
                             stats=st, blocks=t(cuda.row_blocks(kb, kl)))
    o_s, f_s = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), row_ptr=t(rp), key_idx=t(ki))
    torch.cuda.synchronize()
    s = st.cpu().numpy()
    assert s[7] == int(kl.sum()), "the tensor-core kernel did not run"
    assert s[5] == int(kl.sum() + rp[-1])
    assert not f_tc.any().item() and torch.equal(f_tc, f_s)
    assert torch.equal(o_tc, o_s)
    out = o_tc.cpu().numpy().view(np.uint16)
    for r in (0, 5, nodes - 1, nodes + 7):
        keys = np.concatenate([np.arange(P), tails[r]])
        assert np.array_equal(out[r], exact.attention_row(Q[r], K[keys], V[keys], alpha)), r


def test_tensor_core_prefill_fp32_output(ea):
    """fp32 outputs from the tensor-core prefill kernel equal the CUDA-core kernel's and the
    oracle's."""
    import torch

    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(3232)
    S = 260
    Q, K, V, kb, kl = _causal_case(rng, S, "outlier", "wide")
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    st = torch.zeros(12, dtype=torch.int64, device=dev)
    o_tc, f_tc = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), stats=st, out="fp32",
                             blocks=t(cuda.row_blocks(kb, kl)))
    o_s, f_s = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), out="fp32")
    torch.cuda.synchronize()
    assert st.cpu().numpy()[7] == int(kl.sum()), "the tensor-core kernel did not run"
    assert torch.equal(f_tc, f_s) and torch.equal(o_tc, o_s)
    out = o_tc.cpu().numpy().view(np.uint32)
    for r in (0, 9, S - 1, 2 * S - 1):
        L = int(kl[r])
        exp = exact.attention_row(Q[r], K[:L], V[:L], alpha, out="fp32")
        assert np.array_equal(out[r], np.asarray(exp).view(np.uint32)), r


def test_weight_exponent_spread_is_a_domain_error(ea):
    """A row whose logits span more than 2^20 (so its weights' exponents do) is a domain error in
    the reference (reference.py:30, 116-118), also when the small weights are negligible: every
    tier-1 path must flag it, not round it."""
    import torch

    from exactattention_b200 import cuda
    from oracle import exact

    f2b = lambda x: np.uint16(exact.f32_to_bits(np.float32(x)) >> 16)  # noqa: E731
    rng = np.random.default_rng(90)
    n, rows = 300, 16
    K, V = bf16(rng, (n, 128)), bf16(rng, (n, 128))
    Q = bf16(rng, (rows, 128))
    Q[:, 0] = f2b(64.0)
    K[:, 0] = 0
    K[150, 0] = f2b(-262144.0)  # t ~ -2^21 for every row that sees key 150
    kb = np.zeros(rows, np.int64)
    kl = np.array([100, 200, 300, 151] * 4, np.int64)
    sees = kl > 150
    for r in (0, 1):
        L = int(kl[r])
        try:
            exact.attention_row(Q[r], K[:L], V[:L], ea.default_alpha(128))
            assert not sees[r]
        except exact.ExactAttentionDomainError:
            assert sees[r]
    dev = torch.device("cuda")
    t = lambda x: torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)  # noqa: E731
    alpha = ea.default_alpha(128)
    paths = {
        "simt": dict(),
        "tc_prefill": dict(blocks=t(cuda.row_blocks(kb, kl))),
        "decode": dict(segments=t(cuda.row_segments(kb)), splits=2),
    }
    for name, extra in paths.items():
        o, f = cuda.launch(t(Q), t(K), t(V), alpha, kv_base=t(kb), kv_len=t(kl), **extra)
        torch.cuda.synchronize()
        assert np.array_equal(f.cpu().numpy() == 2, sees), name
        assert not o[torch.from_numpy(sees).to(dev)].any().item(), name
