"""The CPU oracle (oracle/exact.py) pinned to the reference's golden vectors and known answers.
Runs without a GPU."""

import hashlib
import json
import math
import os

import numpy as np
import pytest

from oracle import exact

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_config1_sha():
    z = np.load(os.path.join(GOLDEN, "c1.npz"))
    out = exact.attention(z["q"], z["k"], z["v"], z["alpha"])
    assert sha(out) == "27b27a491d2064580a707b042c162d42e3a5f2ca4232043d3de870c840922843"
    assert out[0][:8].tolist() == [48621, 15972, 48697, 48181, 15981, 48787, 15665, 48432]
    assert np.array_equal(exact.attention(z["q"], z["k"], z["v"], z["alpha"], out="fp32").view(np.uint32),
                          z["out32"].view(np.uint32))


def test_config1_inputs_regenerate():
    from exactattention_b200 import workloads

    z = np.load(os.path.join(GOLDEN, "c1.npz"))
    q, k, v, a = workloads.c1()
    assert np.array_equal(q, z["q"]) and np.array_equal(k, z["k"]) and np.array_equal(v, z["v"])
    assert a == z["alpha"]


def test_small_cases():
    z = np.load(os.path.join(GOLDEN, "small_cases.npz"))
    for i in range(int(z["count"])):
        key = f"case{i}"
        fmt = str(z[key + "_fmt"])
        out = exact.attention(z[key + "_q"], z[key + "_k"], z[key + "_v"], z[key + "_alpha"], mask=z[key + "_mask"],
                              out=fmt)
        assert np.array_equal(out.view(np.uint8), z[key + "_out"].view(np.uint8)), key


def test_default_alpha():
    assert exact.default_alpha(128) == np.float32(np.log2(np.e) / np.sqrt(128))
    assert exact.f32_to_bits(exact.default_alpha(64)) == 0x3E38AA3B
    assert exact.f32_to_bits(exact.default_alpha(128)) == 0x3E0293EE
    from exactattention_b200.formats import default_alpha

    for d in (16, 32, 64, 96, 128, 256):
        assert default_alpha(d) == exact.default_alpha(d)


def test_exp2_known_answers():
    z = np.load(os.path.join(GOLDEN, "exp2_kat.npz"))
    for t, M, E in zip(z["t"].tolist(), z["M"].tolist(), z["E"].tolist()):
        assert exact.exp2_rn24_f32(t) == (M, E), t


def test_exp2_integer_t_is_exact_power_of_two():
    for n in [-200, -1, 0, 1, 5, 127, 300]:
        assert exact.exp2_rn24(n, 0) == (1 << 23, n - 23)


@pytest.mark.parametrize("seed", range(2))
def test_exp2_matches_highprec(seed):
    """Independent of the oracle's own interval code: mpmath at 400 bits (the reference's
    test_oracle_matches_highprec)."""
    from mpmath import mp, mpf, power

    rng = np.random.default_rng(seed)
    for t in np.float32(rng.uniform(-80, 80, size=200)).tolist():
        with mp.workprec(400):
            y = power(2, mpf(t))
            n = math.floor(t)
            q = int(mp.floor(y / mpf(2) ** n * 2 ** 23 + mpf("0.5")))
        e = n - 23
        if q == 1 << 24:
            q, e = q >> 1, e + 1
        assert exact.exp2_rn24_f32(t) == (q, e), t


def test_round_ratio_known_answers():
    z = np.load(os.path.join(GOLDEN, "round_kat.npz"))
    for (a, b, E, is32), val, ovf in zip(z["abEf"].tolist(), z["val"].tolist(), z["ovf"].tolist()):
        num, den = (a << E, b) if E >= 0 else (a, b << -E)
        fmt = exact.FP32 if is32 else exact.BF16
        try:
            m, e = exact.round_ratio(num, den, fmt)
            assert not ovf and (m * 2.0 ** e if m else 0.0) == val
        except exact.ExactAttentionDomainError:
            assert ovf


def test_rejects_nan():
    from gen import bf16

    rng = np.random.default_rng(3)
    q, k = bf16(rng, 16), bf16(rng, (3, 16))
    k[1, 2] = 0x7FC0
    with pytest.raises(exact.ExactAttentionDomainError):
        exact.attention_row(q, k, bf16(rng, (3, 16)), exact.default_alpha(16))


def test_empty_set_is_zero():
    from gen import bf16

    rng = np.random.default_rng(2)
    out = exact.attention_row(bf16(rng, 16), np.zeros((0, 16), np.uint16), np.zeros((0, 8), np.uint16),
                              exact.default_alpha(16))
    assert np.array_equal(out, np.zeros(8, np.uint16))


def test_bf16_out_is_rounding_of_exact_ratio():
    """A single rounding of N/Z (the reference's test_bf16_out_is_rounding_of_exact_ratio)."""
    from fractions import Fraction

    from exactattention_b200.formats import bf16_bits_to_float32
    from gen import bf16

    rng = np.random.default_rng(7)
    q, k, v = bf16(rng, 16), bf16(rng, (40, 16)), bf16(rng, (40, 8))
    tr = exact.row_trace(q, k, v, exact.default_alpha(16))
    Zm, Ze = tr["Z"]
    for c, (Nm, Ne) in enumerate(tr["N"]):
        ratio = Fraction(Nm) * Fraction(2) ** Ne / (Fraction(Zm) * Fraction(2) ** Ze)
        o = int(tr["out"][c])
        got = Fraction(float(bf16_bits_to_float32(np.uint16(o))))
        for nb in (o + 1, o - 1 if o & 0x7FFF else o):
            assert abs(got - ratio) <= abs(Fraction(float(bf16_bits_to_float32(np.uint16(nb)))) - ratio)


def test_fixture_heads_via_reference_kernel():
    """oracle/ref.py (the reference's own C++ kernel, built from its sources) reproduces the
    recorded SHA-256 of the real-activation fixture heads. Skipped where it was not built."""
    from oracle import ref

    if not ref.available():
        pytest.skip("oracle/_ref not built")
    z = np.load(os.path.join(GOLDEN, "qwen3_heads.npz"))
    exp = json.load(open(os.path.join(GOLDEN, "qwen3_heads.json")))
    key = "27_11"
    q, k, v, a = z["q_" + key], z["k_" + key], z["v_" + key], np.float32(z["alpha_" + key])
    L = 512  # the first 512 causal rows: a prefix of the fixture, cheap on any CPU
    rp = np.concatenate([[0], np.cumsum(np.arange(1, L + 1))]).astype(np.int64)
    ki = np.concatenate([np.arange(n) for n in range(1, L + 1)]).astype(np.int64)
    out, flags = ref.attention_ref(q[:L], k, v, a, rp, ki, splits=4)
    rows = [0, 1, 100, 511]
    for r in rows:
        assert np.array_equal(out[r], exact.attention_row(q[r], k[:r + 1], v[:r + 1], a))
    assert exp["heads"][key]["rows"] == 2048


def test_reference_kernel_matches_exact_on_random_rows():
    from gen import KINDS, bf16
    from oracle import ref

    if not ref.available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(21)
    for kind in KINDS:
        Q, K, V = bf16(rng, (3, 64), kind), bf16(rng, (50, 64), kind), bf16(rng, (50, 32), "wide")
        a = exact.default_alpha(64)
        got, _ = ref.attention_ref(Q, K, V, a, splits=3)
        assert np.array_equal(got, exact.attention(Q, K, V, a)), kind
