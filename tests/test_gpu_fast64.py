"""The binary64 fast paths of the per-pair roundings against their exact integer evaluations, on
the device (B200): a certified fast result must equal the integer one bit for bit, and nearly
every case must certify (the rest take the integer path inside the kernels)."""

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("start,stride,n", [
    (0x00000000, 1, 1 << 24),        # the smallest logits: w = 1, then the first binades above 2^-27
    (0x3F000000, 1, 1 << 26),        # |t| in [0.5, 4): every fp32 pattern, both signs
    (0x41000000, 1, 1 << 25),        # |t| in [8, 32)
    (0x12345, 97, 1 << 28),          # a stride through the whole range |t| < 2^22
])
def test_weight_fast_path_matches_integer(start, stride, n):
    from exactattention_b200 import cuda

    cases, cert, bad, what = cuda.selftest_fast64(0, start, n, stride)
    assert cases == n
    assert bad == 0, hex(what)
    assert cert >= cases - cases // 10000


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_logit_fast_path_matches_integer(seed):
    from exactattention_b200 import cuda

    n = 1 << 26
    cases, cert, bad, what = cuda.selftest_fast64(1, seed, n)
    assert cases == n
    assert bad == 0, what
    # not certified: results outside the normal fp32 range, exact ties (short scores times alpha
    # often have exactly 25 significant bits), and values within 4 ulps of a midpoint
    assert cert >= cases * 0.95


@pytest.mark.parametrize("mode", [2, 3])  # 3: through one shared reciprocal of the divisor
@pytest.mark.parametrize("seed", [4, 5])
def test_ratio_fast_path_matches_integer(seed, mode):
    from exactattention_b200 import cuda

    n = 1 << 24
    cases, cert, bad, what = cuda.selftest_fast64(mode, seed, n)
    assert cases == n
    assert bad == 0, what
    assert cert >= cases * 0.9  # the rest: results near the subnormal or overflow range, near midpoints
