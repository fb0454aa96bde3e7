"""alpha_for (the reference's validate_model.alpha_for): RN_fp32(scaling / ln 2), checked against
exact rational arithmetic and default_alpha (CPU)."""

from fractions import Fraction

import numpy as np

from exactattention_b200.formats import alpha_for, default_alpha


def _rn32(x: Fraction) -> np.float32:
    # RN-even of a positive rational into fp32 by exact integer arithmetic
    e = x.numerator.bit_length() - x.denominator.bit_length()
    while Fraction(2) ** e > x:
        e -= 1
    while Fraction(2) ** (e + 1) <= x:
        e += 1
    scaled = x / Fraction(2) ** (e - 23)
    q, r = divmod(scaled.numerator, scaled.denominator)
    if 2 * r > scaled.denominator or (2 * r == scaled.denominator and q & 1):
        q += 1
    return np.float32(q * 2.0 ** (e - 23))


# ln 2 to 60 digits (a constant of the test: any 60-digit value decides these cases)
LN2 = Fraction("0.693147180559945309417232121458176568075500134360255254120680")


def test_alpha_for_matches_exact_ratio():
    for scaling in (128 ** -0.5, 64 ** -0.5, 0.1, 0.125, 1.0, 3.0e-3):
        assert alpha_for(scaling) == _rn32(Fraction(scaling) / LN2), scaling


def test_alpha_for_equals_default_alpha_for_power_of_four_dims():
    # 1/sqrt(d) is exact in binary for d = 4^k, so the two routes must agree
    for d in (64, 256, 16):
        assert alpha_for(float(d) ** -0.5) == default_alpha(d)
