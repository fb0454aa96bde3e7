"""The device numerics (exactattention_b200/csrc/ea_numerics.h), built for the host by
tests/probe/numerics_probe.cpp, against the exact oracle. Runs without a GPU."""

import ctypes

import numpy as np
import pytest

from gen import KINDS, bf16
from oracle import exact

u64, i64, i32, u32 = ctypes.c_uint64, ctypes.c_int64, ctypes.c_int, ctypes.c_uint32


@pytest.fixture(scope="module")
def P(probe_lib):
    L = probe_lib
    L.probe_exp2_q63.restype = u64
    L.probe_exp2_q63.argtypes = [u64]
    L.probe_exp2_q127.argtypes = [u64, ctypes.POINTER(u64), ctypes.POINTER(u64)]
    L.probe_weight.argtypes = [i32, u64, i32, i32, ctypes.POINTER(u32), ctypes.POINTER(i64)]
    L.probe_round_ratio64.restype = u32
    L.probe_round_ratio64.argtypes = [u64, u64, i32, i32, i32, ctypes.POINTER(i32)]
    L.probe_logit_interval.argtypes = [i64, u64, i32, u32, ctypes.POINTER(u32)]
    L.probe_logit_exact.argtypes = [ctypes.c_void_p, ctypes.c_void_p, i32, u32, ctypes.POINTER(u32)]
    L.probe_logit_exact64.argtypes = [i64, i32, u32, ctypes.POINTER(u32)]
    L.probe_logit_i128.argtypes = [i64, u64, i32, u32, ctypes.POINTER(u32)]
    L.probe_certify_ratio.argtypes = [i64, u64, i64, i64, u64, i64, i32, ctypes.POINTER(u32)]
    return L


def _bits(m, e, fp32=True):
    if m == 0:
        return 0
    b = exact.f32_to_bits(np.float32(m * 2.0 ** e))
    return b if fp32 else b >> 16


def test_exp2_error_bound(P):
    """|Y - 2^f 2^63| <= 7.4 units (the analysed bound, EXP2_ERR = 8) on random f and every table
    boundary; the 128-bit evaluation within 64 units of 2^-127."""
    from mpmath import mp, mpf

    rng = np.random.default_rng(7)
    F = [int(x) for x in rng.integers(0, 1 << 50, 1500)]
    F += [(a << 42) + (b << 34) + c for a in (0, 1, 128, 255) for b in (0, 1, 200, 255) for c in (0, 1, (1 << 34) - 1)]
    F += [0, 1, (1 << 50) - 1]
    worst = worst2 = 0.0
    with mp.workprec(320):
        for f in F:
            y = P.probe_exp2_q63(f)
            worst = max(worst, abs(float(mpf(y) - mp.power(2, mpf(f) / 2 ** 50 + 63))))
            hi, lo = u64(), u64()
            P.probe_exp2_q127(f, hi, lo)
            y2 = (hi.value << 64) | lo.value
            worst2 = max(worst2, abs(float(mpf(y2) - mp.power(2, mpf(f) / 2 ** 50 + 127))))
    assert worst <= 7.4, worst
    assert worst2 <= 64, worst2


@pytest.mark.parametrize("wide", [0, 1])
def test_weights_match_oracle(P, wide):
    rng = np.random.default_rng(300 + wide)
    ts = np.float32(np.concatenate([
        rng.uniform(-60, 60, 8000), rng.uniform(-1e-6, 1e-6, 800),
        np.float32(2.0) ** rng.uniform(-40, -20, 400) * rng.choice([-1, 1], 400),
        np.arange(-40, 40) + rng.uniform(-1e-7, 1e-7, 80), rng.uniform(-1e4, 1e4, 800),
        [0.0, -0.0, 1.0, -1.0, 2.0 ** -27, -(2.0 ** -27), 2.0 ** -28, np.nextafter(np.float32(1), 0), 2.0 ** 29,
         -(2.0 ** 29), 2.0 ** 30, -(2.0 ** 31)]]))
    risky = 0
    for t in ts.tolist():
        m, e = exact.decode_fp32(t)
        M, E = u32(), i64()
        st = P.probe_weight(int(m < 0), abs(m), e, wide, M, E)
        if abs(t) >= 2 ** 30:
            assert st == 2
            continue
        if st == 1:
            risky += 1
            continue
        assert st == 0 and (M.value, E.value) == exact.exp2_rn24(m, e), t
    assert risky <= 2


def test_round_ratio64(P):
    rng = np.random.default_rng(5)
    for _ in range(6000):
        a = max(1, int(rng.integers(1, 2 ** 62)) >> int(rng.integers(0, 62)))
        b = max(1, int(rng.integers(1, 2 ** 62)) >> int(rng.integers(0, 62)))
        sh, neg = int(rng.integers(-200, 150)), int(rng.integers(0, 2))
        for fp32 in (0, 1):
            ov = i32()
            got = P.probe_round_ratio64(a, b, sh, neg, fp32, ov)
            num, den = (a << sh, b) if sh >= 0 else (a, b << -sh)
            try:
                m, e = exact.round_ratio(-num if neg else num, den, exact.FP32 if fp32 else exact.BF16)
                assert not ov.value and got == _bits(m, e, fp32)
            except exact.ExactAttentionDomainError:
                assert ov.value


def test_logit_interval_exact_point(P):
    rng = np.random.default_rng(6)
    a = exact.default_alpha(128)
    am, ae = exact.decode_fp32(a)
    for _ in range(6000):
        acc = int(rng.integers(-2 ** 62, 2 ** 62)) >> int(rng.integers(0, 62))
        sexp = int(rng.integers(-300, 100))
        tb = u32()
        st = P.probe_logit_interval(acc, 0, sexp, exact.f32_to_bits(a), tb)
        try:
            m, e = exact.round_dyadic(am * acc, ae + sexp, exact.FP32) if acc else (0, 0)
            assert st == 0 and tb.value == _bits(m, e)
        except exact.ExactAttentionDomainError:
            assert st == 2


def test_logit_exact64_matches_oracle(P):
    """The exact-product rounding of a 64-bit score, including the subnormal range, ties and
    overflow."""
    rng = np.random.default_rng(12)
    for alpha in (exact.default_alpha(128), np.float32(0.0883883), np.float32(-3.5e-39), np.float32(1.7e38)):
        am, ae = exact.decode_fp32(alpha)
        ab = exact.f32_to_bits(alpha)
        for _ in range(4000):
            acc = int(rng.integers(-2 ** 62, 2 ** 62)) >> int(rng.integers(0, 62))
            if rng.random() < 0.2:   # low bits that only matter as sticky
                acc = (acc >> 20 << 20) | int(rng.integers(0, 2))
            sexp = int(rng.integers(-330, 120))
            tb = u32()
            st = P.probe_logit_exact64(acc, sexp, ab, tb)
            try:
                m, e = exact.round_dyadic(am * acc, ae + sexp, exact.FP32) if acc and am else (0, 0)
                assert st == 0 and tb.value == _bits(m, e), (acc, sexp)
            except exact.ExactAttentionDomainError:
                assert st == 2


def _carry_cases(am, n, seed):
    """Scores whose product with am rounds differently when the bits of the score below its top
    40 are dropped before the multiplication (kept only as a sticky bit): the dropped part times
    am carries across the rounding midpoint. These need the exact product."""
    rng = np.random.default_rng(seed)
    out = []
    a = abs(am)
    while len(out) < n:
        acc = int(rng.integers(1 << 54, 1 << 62)) | 1
        drop = acc.bit_length() - 40
        top = acc >> drop
        p_top, p_ex = top * a, acc * a
        sh_t = p_top.bit_length() - 24
        sh_e = p_ex.bit_length() - 24
        rt = (p_top >> sh_t) + (((p_top >> (sh_t - 1)) & 1) if sh_t > 0 else 0)
        re = (p_ex >> sh_e) + (((p_ex >> (sh_e - 1)) & 1) if sh_e > 0 else 0)
        if rt << (sh_t + drop) != re << sh_e:
            out.append(acc)
    return out


def test_logit_exact64_carry_across_midpoint(P):
    alpha = exact.default_alpha(128)
    am, ae = exact.decode_fp32(alpha)
    for acc in _carry_cases(am, 6, 21):
        for sg in (1, -1):
            tb = u32()
            st = P.probe_logit_exact64(sg * acc, -40, exact.f32_to_bits(alpha), tb)
            m, e = exact.round_dyadic(am * sg * acc, ae - 40, exact.FP32)
            assert st == 0 and tb.value == _bits(m, e), acc
            S = sg * acc << 50
            st = P.probe_logit_i128(S >> 64, S & ((1 << 64) - 1), -90, exact.f32_to_bits(alpha), tb)
            m, e = exact.round_dyadic(am * S, ae - 90, exact.FP32)
            assert st == 0 and tb.value == _bits(m, e), acc


def test_logit_i128_matches_oracle(P):
    rng = np.random.default_rng(13)
    for alpha in (exact.default_alpha(128), np.float32(-3.5e-39), np.float32(1.7e38)):
        am, ae = exact.decode_fp32(alpha)
        for _ in range(3000):
            S = int(rng.integers(-2 ** 62, 2 ** 62)) << int(rng.integers(0, 62))
            S += int(rng.integers(-3, 3))
            S >>= int(rng.integers(0, 100))
            E = int(rng.integers(-400, 50))
            tb = u32()
            st = P.probe_logit_i128(S >> 64, S & ((1 << 64) - 1), E, exact.f32_to_bits(alpha), tb)
            try:
                m, e = exact.round_dyadic(am * S, ae + E, exact.FP32) if S and am else (0, 0)
                assert st == 0 and tb.value == _bits(m, e), (S, E)
            except exact.ExactAttentionDomainError:
                assert st == 2


def test_logit_interval_soundness(P):
    """A certified interval returns the exact logit of every point inside it."""
    rng = np.random.default_rng(8)
    a = exact.default_alpha(64)
    am, ae = exact.decode_fp32(a)
    certified = 0
    for _ in range(3000):
        acc = int(rng.integers(-2 ** 50, 2 ** 50))
        err = int(rng.integers(0, 1 << int(rng.integers(0, 20))))
        sexp = int(rng.integers(-60, -20))
        tb = u32()
        st = P.probe_logit_interval(acc, err, sexp, exact.f32_to_bits(a), tb)
        if st != 0:
            continue
        certified += 1
        for x in (acc - err, acc + err, acc + int(rng.integers(-err, err + 1))):
            m, e = exact.round_dyadic(am * x, ae + sexp, exact.FP32) if x else (0, 0)
            assert tb.value == _bits(m, e)
    assert certified > 1000


@pytest.mark.parametrize("kind", KINDS)
def test_exact_logit(P, kind):
    rng = np.random.default_rng(hash(kind) & 0xFFFF)
    a = exact.default_alpha(128)
    am, ae = exact.decode_fp32(a)
    for _ in range(150):
        d = int(rng.choice([16, 64, 128, 256]))
        q, k = bf16(rng, d, kind), bf16(rng, d, kind)
        tb = u32()
        st = P.probe_logit_exact(q.ctypes.data, k.ctypes.data, d, exact.f32_to_bits(a), tb)
        qm, qe, _ = exact.decode_bf16_np(q)
        km, ke, _ = exact.decode_bf16_np(k)
        S, E = exact.exact_score(qm, qe, km, ke)
        m, e = exact.round_dyadic(am * S, ae + E, exact.FP32) if S else (0, 0)
        assert st == 0 and tb.value == _bits(m, e)


def test_certify_ratio_soundness(P):
    """When both ends of [N, N+Nerr]/[Z, Z+Zerr] round alike, every ratio inside rounds to it."""
    rng = np.random.default_rng(10)
    hits = 0
    for _ in range(3000):
        Z = int(rng.integers(1, 2 ** 61))
        Ze = int(rng.integers(0, 1 << int(rng.integers(0, 30))))
        N = int(rng.integers(-2 ** 61, 2 ** 61))
        Ne = int(rng.integers(0, 1 << int(rng.integers(0, 30))))
        nu, zu = int(rng.integers(-80, 0)), int(rng.integers(-80, 0))
        for fp32 in (0, 1):
            bits = u32()
            if not P.probe_certify_ratio(N, Ne, nu, Z, Ze, zu, fp32, bits):
                continue
            hits += 1
            fmt = exact.FP32 if fp32 else exact.BF16
            for n_, z_ in ((N, Z), (N + Ne, Z + Ze), (N + Ne // 2, Z + Ze // 3)):
                sh = nu - zu
                num, den = (n_ << sh, z_) if sh >= 0 else (n_, z_ << -sh)
                m, e = exact.round_ratio(num, den, fmt)
                assert bits.value == _bits(m, e, fp32)
    assert hits > 1000
