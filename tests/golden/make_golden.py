"""Writes the golden fixtures under tests/golden/ from the reference itself.

Run where a checkout of the reference repository is available; its path must be given in
EA_REFERENCE_DIR (there is no default):

    EA_REFERENCE_DIR=<checkout> python tests/golden/make_golden.py            # small fixtures (seconds)
    EA_REFERENCE_DIR=<checkout> python tests/golden/make_golden.py --configs  # + SHA-256 of the full synthetic configs (minutes)

Outputs
  c1.npz              config 1 (README example): inputs and the reference's exact output
  qwen3_heads.npz     the reference's two real-activation fixture heads (fixtures/*.npz) and
  qwen3_heads.json    their recorded SHA-256 (fixtures/expected_sha256.json)
  small_cases.npz     random rows of every generator kind (tests/gen.py of the reference) with
                      the reference's exact outputs (reference.attention), bf16 and fp32
  exp2_kat.npz        fp32 logits and the reference oracle's RN24(2^t) (exp2_weight_oracle)
  round_kat.npz       RN of random ratios by the reference's round_rational
  configs.json        SHA-256 of configs 2-5 computed by the reference's C++ kernel with exact
                      fallback (oracle/ref.py) on the generators of exactattention_b200/workloads.py
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
REF = os.environ.get("EA_REFERENCE_DIR", "")
if not REF or not os.path.isdir(os.path.join(REF, "src", "exactattn")):
    sys.exit("make_golden.py: set EA_REFERENCE_DIR to a checkout of the reference repository")
REF = os.path.abspath(REF)
sys.path.insert(0, os.path.join(REF, "src"))
sys.path.insert(0, os.path.join(REF, "tests"))
sys.path.insert(0, REPO)


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_small() -> None:
    import exactattn
    from exactattn import exp2 as rexp2, formats as rformats
    from gen import KINDS, bf16

    # config 1 (README.md example of the reference)
    rng = np.random.default_rng(0)
    q = exactattn.float_to_bf16_bits(rng.standard_normal((2, 64)))
    k = exactattn.float_to_bf16_bits(rng.standard_normal((100, 64)))
    v = exactattn.float_to_bf16_bits(rng.standard_normal((100, 64)))
    alpha = exactattn.default_alpha(64)
    out = exactattn.attention(q, k, v, alpha)
    out32 = exactattn.attention(q, k, v, alpha, out="fp32")
    np.savez_compressed(os.path.join(HERE, "c1.npz"), q=q, k=k, v=v, alpha=np.float32(alpha), out=out,
                        out32=out32)
    print("c1", sha(out))

    # real-activation fixture heads
    z = np.load(os.path.join(REF, "fixtures", "qwen3_0.6b_heads.npz"))
    np.savez_compressed(os.path.join(HERE, "qwen3_heads.npz"), **{k_: z[k_] for k_ in z.files})
    exp = json.load(open(os.path.join(REF, "fixtures", "expected_sha256.json")))
    json.dump(exp, open(os.path.join(HERE, "qwen3_heads.json"), "w"), indent=1)

    # random rows of every kind, dense / masked, bf16 / fp32
    cases = {}
    rng = np.random.default_rng(1234)
    idx = 0
    for kind in KINDS:
        for vkind in ("normal", "wide", "dupes"):
            for out_fmt in ("bf16", "fp32"):
                d = int(rng.choice([16, 32, 64, 128]))
                dv = int(rng.choice([8, 32, 64]))
                n = int(rng.integers(1, 90))
                r = int(rng.integers(1, 4))
                Q, K, V = bf16(rng, (r, d), kind), bf16(rng, (n, d), kind), bf16(rng, (n, dv), vkind)
                mask = rng.random((r, n)) < 0.7 if idx % 2 else None
                a = exactattn.default_alpha(d)
                res = exactattn.attention(Q, K, V, a, mask=mask, out=out_fmt)
                key = f"case{idx}"
                cases[key + "_q"], cases[key + "_k"], cases[key + "_v"] = Q, K, V
                cases[key + "_mask"] = mask if mask is not None else np.ones((r, n), bool)
                cases[key + "_alpha"] = np.float32(a)
                cases[key + "_out"] = res
                cases[key + "_fmt"] = np.array(out_fmt)
                idx += 1
    cases["count"] = np.array(idx)
    np.savez_compressed(os.path.join(HERE, "small_cases.npz"), **cases)
    print("small cases", idx)

    # exp2 known answers
    rng = np.random.default_rng(77)
    ts = np.float32(np.concatenate([rng.uniform(-80, 80, 4000), rng.uniform(-1e-6, 1e-6, 300),
                                    np.arange(-40, 40) + rng.uniform(-1e-7, 1e-7, 80),
                                    rng.uniform(-1e4, 1e4, 300), [0.0, 1.0, -1.0, 2.0 ** -27, -(2.0 ** -27)]]))
    M, E = zip(*[rexp2.exp2_weight_oracle(float(t)) for t in ts])
    np.savez_compressed(os.path.join(HERE, "exp2_kat.npz"), t=ts, M=np.array(M, np.int64), E=np.array(E, np.int64))

    # ratio rounding known answers (formats.round_rational)
    rng = np.random.default_rng(78)
    rows = []
    for _ in range(4000):
        a = int(rng.integers(1, 2 ** 62)) >> int(rng.integers(0, 60))
        b = int(rng.integers(1, 2 ** 62)) >> int(rng.integers(0, 60))
        a, b = max(a, 1), max(b, 1)
        E = int(rng.integers(-200, 150))
        for fmt, is32 in ((rformats.FP32, 1), (rformats.BF16, 0)):
            num, den = (a << E, b) if E >= 0 else (a, b << -E)
            try:
                m, e = rformats.round_rational(num, den, fmt)
                val = float(np.float32(m * 2.0 ** e)) if m else 0.0
                rows.append((a, b, E, is32, val, 0))
            except rformats.ExactAttentionDomainError:
                rows.append((a, b, E, is32, 0.0, 1))
    arr = np.array([r[:4] for r in rows], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "round_kat.npz"), abEf=arr, val=np.array([r[4] for r in rows]),
                        ovf=np.array([r[5] for r in rows], np.int8))


def make_configs() -> None:
    from exactattention_b200 import workloads
    from oracle import ref

    res = {}
    for name in ("c2", "c3", "c4", "c5"):
        t0 = time.time()
        h = workloads.reference_sha(name, ref.attention_ref)
        res[name] = h
        print(name, h, f"{time.time() - t0:.1f}s", flush=True)
        json.dump(res, open(os.path.join(HERE, "configs.json"), "w"), indent=1)


if __name__ == "__main__":
    if "--configs-only" not in sys.argv:
        make_small()
    if "--configs" in sys.argv or "--configs-only" in sys.argv:
        make_configs()
