"""Portable bit-identity check on the reference's two real-activation heads.

    python -m exactattention_b200.fixture check [--backend cuda|torch:cuda] [--only 0_0]

Every causal row of each head goes through the chosen backend; the SHA-256 of the bf16 output
bits must equal the one the reference recorded (its scripts/fixture.py check, fixtures/
expected_sha256.json). Prints `ALL MATCH` and exits 0 when every head matches.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "..", "tests", "golden")


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def run_backend(backend: str, q, k, v, alpha):
    L = q.shape[0]
    kv_len = np.arange(1, L + 1)
    if backend == "cuda":
        from .cuda import attention_cuda

        row_ptr = np.concatenate([[0], np.cumsum(kv_len)]).astype(np.int64)
        key_idx = np.concatenate([np.arange(n) for n in kv_len]).astype(np.int64)
        return attention_cuda(q, k, v, alpha, row_ptr, key_idx, splits=8, tile=64)
    kind, _, dev = backend.partition(":")
    if kind == "torch":
        from .torch_impl import attention_torch

        mask = np.tril(np.ones((L, L), bool))
        return attention_torch(q, k, v, alpha, mask, device=dev or "cuda")
    raise ValueError(f"unknown backend {backend!r} (cuda or torch:cuda)")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["check"])
    ap.add_argument("--backend", default="cuda")
    ap.add_argument("--only", default=None)
    args = ap.parse_args(argv)
    z = np.load(os.path.join(GOLDEN, "qwen3_heads.npz"))
    expected = json.load(open(os.path.join(GOLDEN, "qwen3_heads.json")))
    only = set(args.only.split(",")) if args.only else None
    ok = True
    for key, info in expected["heads"].items():
        if only is not None and key not in only:
            continue
        q, k, v, alpha = z[f"q_{key}"], z[f"k_{key}"], z[f"v_{key}"], np.float32(z[f"alpha_{key}"])
        t0 = time.perf_counter()
        out, flags = run_backend(args.backend, q, k, v, alpha)
        dt = time.perf_counter() - t0
        h = sha(out)
        match = h == info["sha256"]
        ok &= match
        extra = ""
        if args.backend == "cuda":
            from ._lib import last_host_stats

            st = last_host_stats()
            extra = f", {st['tc_pairs']} of {st['pairs']} pairs on the tensor cores"
        print(f"head {key}: {'MATCH' if match else 'MISMATCH'} sha256 {h[:16]}  ({dt:.2f}s, "
              f"{int((flags != 0).sum())} flagged rows, 0 host fallbacks{extra})", flush=True)
    print("ALL MATCH" if ok else "MISMATCH")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
