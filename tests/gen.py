"""Random bf16 test inputs: the reference's generator kinds (tests/gen.py:10-35 of the reference),
restated: normal, wide (log-uniform 2^-40..2^8), outlier (2% at 30x a 0.05 base), dupes (seven
values: ties and cancellation) and subnormal (x 2^-130)."""

from __future__ import annotations

import numpy as np

from exactattention_b200.formats import float_to_bf16_bits

KINDS = ["normal", "wide", "outlier", "dupes", "subnormal"]


def bf16(rng: np.random.Generator, shape, kind: str = "normal", scale: float = 1.0) -> np.ndarray:
    if kind == "normal":
        x = rng.standard_normal(shape) * scale
    elif kind == "wide":
        x = np.exp2(rng.uniform(-40, 8, size=shape)) * rng.choice([-1.0, 1.0], size=shape)
    elif kind == "outlier":
        x = rng.standard_normal(shape) * 0.05 * scale
        x = np.where(rng.random(shape) < 0.02, rng.standard_normal(shape) * 30 * scale, x)
    elif kind == "dupes":
        x = rng.choice(np.array([-2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0]) * scale, size=shape)
    elif kind == "heavy":  # 1% of rows scaled by 32 (long-context stress: wide channel ranges)
        x = rng.standard_normal(shape) * scale
        x = x * np.where(rng.random(shape[:1]) < 0.01, 32.0, 1.0).reshape((-1,) + (1,) * (len(shape) - 1))
    elif kind == "subnormal":
        x = rng.standard_normal(shape) * 2.0 ** -130
    else:
        raise ValueError(kind)
    return float_to_bf16_bits(x)
