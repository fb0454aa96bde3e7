"""The fallback tiers and the failure reporting of the device path (B200 only).

Rows that tier 1 cannot certify are rerun on the GPU by tier 2 and, failing that, tier 3; a test
hook forces certified rows out of tier 1 (and tier 2) so that these tiers run on ordinary inputs,
and the bits must not change (the reference drives its fallbacks the same way, by narrowing its
windows: tests/test_certified.py:129-139). A second hook makes the tensor-core kernels' bounded
waits report expiry after their phase completed, which runs the abort path with nothing in
flight: the host-pointer entry points return -5, the device counter records the CTAs, and the
rows are still exact. Nothing here faults or hangs a GPU.
"""

import numpy as np
import pytest

from gen import bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ea(cuda_lib):
    import torch

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    import exactattention_b200 as ea

    return ea


@pytest.fixture
def hooks():
    from exactattention_b200 import _lib

    yield _lib.set_test_hooks
    _lib.set_test_hooks(0, 0, 0)


def _t(x, dev="cuda"):
    import torch

    return torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)


def _prefill_case(rng, S=200, heads=2):
    Q = bf16(rng, (heads * S, 128), "outlier")
    K = bf16(rng, (S, 128), "outlier")
    V = bf16(rng, (S, 128), "normal")
    kb = np.zeros(heads * S, np.int64)
    kl = np.tile(np.arange(1, S + 1, dtype=np.int64), heads)
    return Q, K, V, kb, kl


def _decode_case(rng, n=700, rows=4):
    Q = bf16(rng, (rows, 128), "normal")
    K = bf16(rng, (n, 128), "heavy")
    V = bf16(rng, (n, 128), "heavy")
    return Q, K, V, np.zeros(rows, np.int64), np.full(rows, n, np.int64)


def _launch(cuda, Q, K, V, kb, kl, alpha, st, mode, splits=1):
    kw = dict(kv_base=_t(kb), kv_len=_t(kl), stats=st, splits=splits)
    if mode == "prefill":
        kw["blocks"] = _t(cuda.row_blocks(kb, kl))
    elif mode == "decode":
        kw["segments"] = _t(cuda.row_segments(kb))
    o, f = cuda.launch(_t(Q), _t(K), _t(V), alpha, **kw)
    return o.cpu().numpy().view(np.uint16), f.cpu().numpy()


@pytest.mark.parametrize("mode,splits", [("prefill", 1), ("decode", 3), ("simt", 2)])
def test_forced_rows_keep_their_bits(ea, hooks, mode, splits):
    """Rows forced out of tier 1 (then also out of tier 2) come back with the same bits."""
    from exactattention_b200 import cuda

    rng = np.random.default_rng(11)
    Q, K, V, kb, kl = _prefill_case(rng) if mode != "decode" else _decode_case(rng)
    alpha = ea.default_alpha(128)
    st0 = cuda.new_stats()
    base, f0 = _launch(cuda, Q, K, V, kb, kl, alpha, st0, mode, splits)
    assert not f0.any()
    rows = Q.shape[0]
    stride = 3
    forced = len(range(0, rows, stride))
    for tier in (1, 2):
        hooks(stride, tier, 0)
        st = cuda.new_stats()
        out, fl = _launch(cuda, Q, K, V, kb, kl, alpha, st, mode, splits)
        s = st.cpu().numpy()
        assert not fl.any()
        assert np.array_equal(out, base), f"tier {tier}"
        assert s[11] == forced and s[2] >= forced
        if tier == 2:
            assert s[9] >= forced  # tier 2 handed them on to tier 3
        hooks(0, 0, 0)


def test_expired_waits_are_reported_and_rows_stay_exact(ea, hooks):
    """Every bounded wait of the tensor-core kernels reports expiry (after its phase completed):
    the kernels abort, drain, count the CTAs; the rows are recomputed exactly; the synchronous
    host-pointer entry returns -5, which the Python layer reports as a warning."""
    from exactattention_b200 import _lib, cuda
    from oracle import exact

    rng = np.random.default_rng(12)
    alpha = ea.default_alpha(128)
    Qp, Kp, Vp, kbp, klp = _prefill_case(rng, S=130, heads=1)
    Qd, Kd, Vd, kbd, kld = _decode_case(rng, n=300, rows=2)
    ref_p = np.stack([exact.attention_row(Qp[r], Kp[:kl], Vp[:kl], alpha) for r, kl in enumerate(klp)])
    ref_d = np.stack([exact.attention_row(Qd[r], Kd, Vd, alpha) for r in range(2)])
    hooks(0, 0, 1)
    st = cuda.new_stats()
    out_p, f_p = _launch(cuda, Qp, Kp, Vp, kbp, klp, alpha, st, "prefill")
    out_d, f_d = _launch(cuda, Qd, Kd, Vd, kbd, kld, alpha, st, "decode", splits=2)
    s = st.cpu().numpy()
    assert s[8] >= 3, f"expired waits counted: {s[8]}"  # the prefill CTA and both decode CTAs
    assert not f_p.any() and not f_d.any()
    assert np.array_equal(out_p, ref_p) and np.array_equal(out_d, ref_d)
    with pytest.warns(_lib.WaitExpiredWarning):
        out_h, _ = cuda.attention_cuda_ranges(Qd, Kd, Vd, alpha, kbd, kld, splits=2)
    assert np.array_equal(out_h, ref_d)
    hooks(0, 0, 0)
    st2 = cuda.new_stats()
    out_p2, _ = _launch(cuda, Qp, Kp, Vp, kbp, klp, alpha, st2, "prefill")
    assert st2.cpu().numpy()[8] == 0 and np.array_equal(out_p2, ref_p)


@pytest.mark.parametrize("dv", [320, 512])
def test_value_rows_wider_than_256(ea, dv):
    """More than 256 value channels: every row on the wide tier, bits equal to the oracle (the
    reference's CPU entry accepts any dv)."""
    from exactattention_b200 import cuda
    from oracle import exact

    rng = np.random.default_rng(dv)
    Q, K, V = bf16(rng, (5, 64)), bf16(rng, (90, 64), "outlier"), bf16(rng, (90, dv))
    alpha = ea.default_alpha(64)
    mask = rng.random((5, 90)) < 0.7
    mask[4] = False  # an empty row
    out = ea.attention(Q, K, V, alpha, mask=mask)
    assert np.array_equal(out, exact.attention(Q, K, V, alpha, mask=mask))
    o, f = cuda.launch(_t(Q), _t(K), _t(V), alpha, kv_base=_t(np.zeros(5, np.int64)),
                       kv_len=_t(np.full(5, 90, np.int64)), out="fp32")
    assert not f.cpu().numpy().any()
    ref32 = exact.attention(Q, K, V, alpha, out="fp32")
    assert np.array_equal(o.cpu().numpy().view(np.uint32), ref32.view(np.uint32))


def _golden_configs():
    import json
    import os

    p = os.path.join(os.path.dirname(__file__), "golden", "configs.json")
    return json.load(open(p)) if os.path.exists(p) else {}


@pytest.mark.parametrize("name,stride,tier", [("c5", 64, 1), ("c5", 64, 2), ("c2", 100, 1), ("c2", 100, 2)])
def test_config_with_forced_rows_keeps_sha(ea, hooks, name, stride, tier):
    """About 1% of a full configuration's rows forced out of tier 1 (and tier 2): the SHA-256 of
    the outputs is still the reference's, tier 2 (and tier 3) count their work, and on config 5
    (one forced row of 2^20 keys) the step costs less than twice the clean step (the rows are
    split by key chunks over the whole GPU instead of one block per row)."""
    import hashlib

    import torch

    from exactattention_b200 import cuda, workloads as w

    gold = _golden_configs().get(name)
    if gold is None:
        pytest.skip(f"no golden SHA for {name}")
    case = w.device_case(name)
    splits = 32 if name == "c5" else 1

    def run(st):
        return cuda.launch(case["q"], case["k"], case["v"], case["cfg"].alpha, splits=splits, stats=st, **case["kw"])

    def timed(n=3):
        ts = []
        for _ in range(n):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            run(cuda.new_stats())
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return sorted(ts)[n // 2]

    run(cuda.new_stats())
    clean_ms = timed()
    hooks(stride, tier, 0)
    st = cuda.new_stats()
    out, flags = run(st)
    torch.cuda.synchronize()
    s = st.cpu().numpy()
    forced = len(range(0, case["cfg"].rows, stride))
    assert not flags.any().item()
    assert hashlib.sha256(out.cpu().numpy().view(np.uint16).tobytes()).hexdigest() == gold
    assert s[11] == forced and s[2] == forced
    assert s[10] > 0  # tier 2 ran on the forced rows' keys
    if tier == 2:
        assert s[9] == forced
    forced_ms = timed()
    print(f"{name} forced tier {tier}: clean {clean_ms:.2f} ms, with {forced} forced rows {forced_ms:.2f} ms")
    if name == "c5":
        assert forced_ms < 2 * clean_ms, (clean_ms, forced_ms)


def _row(qhead, kheads, vcol, d=128):
    """One query row whose leading elements are `qhead` against keys whose leading elements are
    kheads[j] (the rest zero) and values v_j[0] = vcol[j], as bf16 bits."""
    import exactattention_b200 as ea

    q = np.zeros((1, d), np.float32)
    k = np.zeros((len(kheads), d), np.float32)
    v = np.zeros((len(kheads), d), np.float32)
    q[0, :len(qhead)] = qhead
    for j, kh in enumerate(kheads):
        k[j, :len(kh)] = kh
    v[:, 0] = vcol
    return ea.float_to_bf16_bits(q), ea.float_to_bf16_bits(k), ea.float_to_bf16_bits(v)


@pytest.mark.parametrize("route", ["prefill", "decode", "forced"])
def test_logits_between_2_30_and_2_62_are_exact(ea, hooks, route):
    """Logits of 2^30 .. 2^62 (weight exponents past int32) send their row from the tensor-core
    kernels to the wide tier, which keeps them exactly: equal to the exact oracle, whether the
    prefill kernel (row blocks) or the decode kernel (a segment) ran tier 1, or the row was
    forced past tiers 1 and 2. Near 2^31 an fp32 logit moves in steps of 256, so two keys tie at
    the top and the third lies ~520 binades below (under the reference's 2^20 spread limit)."""
    import torch

    from exactattention_b200 import cuda
    from oracle import exact

    alpha = ea.default_alpha(128)
    Q, K, V = _row([2.0 ** 17, 1.0], [[2.0 ** 17, 0.0], [2.0 ** 17, 0.0], [2.0 ** 17, -4096.0]], [1.0, 3.0, -2.0])
    Q = np.repeat(Q, 2, axis=0)  # a GQA pair of identical rows
    kb, kl = np.zeros(2, np.int64), np.full(2, 3, np.int64)
    sched = dict(blocks=_t(cuda.row_blocks(kb, kl))) if route == "prefill" else \
        dict(segments=_t(cuda.row_segments(kb)), segment_width=2)
    if route == "forced":
        hooks(1, 2, 0)
    st = torch.zeros(12, dtype=torch.int64, device="cuda")
    out, flags = cuda.launch(_t(Q), _t(K), _t(V), alpha, kv_base=_t(kb), kv_len=_t(kl), max_row_keys=3, stats=st,
                             **sched)
    torch.cuda.synchronize()
    hooks(0, 0, 0)
    assert not flags.any().item()
    exp = exact.attention(Q, K, V, alpha)
    assert exp[0, 0] == 0x4000  # 2.0: the mean of the two tied keys' values
    assert np.array_equal(out.cpu().numpy().view(np.uint16), exp)
    if route != "forced":
        assert int(st[7].item()) == 6  # the pairs ran on the tensor cores first


def test_logits_from_2_62_are_a_domain_error_here(ea):
    """A documented limit of this build: the wide tier keeps weight exponents in int64, so a row
    whose logits reach 2^62 (|q . k| around 2^63, far outside bf16 model activations) is flagged
    as a domain error, where the reference's unbounded Python integers still return its value
    (here 2.0, the mean of the three values)."""
    from oracle import exact

    alpha = ea.default_alpha(128)
    Q, K, V = _row([2.0 ** 40], [[2.0 ** 40]] * 3, [1.0, 2.0, 3.0])
    assert exact.attention(Q, K, V, alpha)[0, 0] == 0x4000  # the reference's answer: 2.0
    with pytest.raises(ea.ExactAttentionDomainError):
        ea.attention(Q, K, V, alpha)


def test_weights_spanning_1300_binades_through_the_wide_tier(ea, hooks):
    """A row whose weights span ~1300 binades (beyond the wide tier's exact 1536-bit window, under
    the reference's 2^20 spread limit), forced through tier 3: the counted truncation still
    certifies it, equal to the exact oracle."""
    from oracle import exact

    alpha = ea.default_alpha(128)
    # t = alpha s: 0, about -326, 0.13 and -1306 for s = 0, -2560, 1, -10240 (alpha = 0.1275):
    # weights 1, 2^-326, 2^0.13, 2^-1306, with the values 1, 2^100, 0.5, 2^-20 the terms span
    # ~1330 binades
    Q, K, V = _row([1.0], [[0.0], [-2560.0], [1.0], [-10240.0]], [1.0, 2.0 ** 100, 0.5, 2.0 ** -20])
    hooks(1, 2, 0)
    out = ea.attention(Q, K, V, alpha)
    hooks(0, 0, 0)
    assert np.array_equal(out, exact.attention(Q, K, V, alpha))
