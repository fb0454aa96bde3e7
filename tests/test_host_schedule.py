"""Host-side scheduling of masks onto the kernels (no GPU): CSR rows of a boolean mask split into
a leading run of consecutive keys plus a tail list, so that causal / prefix / tree masks reach the
tensor-core kernels. The split must describe exactly the same keys."""

import numpy as np
from hypothesis import given
from hypothesis import strategies as st

from exactattention_b200 import cuda


def _csr(mask):
    rp = np.concatenate([[0], np.cumsum(mask.sum(axis=1))]).astype(np.int64)
    ki = (np.concatenate([np.flatnonzero(m) for m in mask]) if mask.size else np.zeros(0)).astype(np.int64)
    return rp, ki


@given(st.integers(1, 12), st.integers(1, 40), st.integers(0, 2 ** 32 - 1), st.sampled_from(["rand", "tree", "causal"]))
def test_split_runs_keeps_every_key(rows, n, seed, kind):
    rng = np.random.default_rng(seed)
    if kind == "rand":
        mask = rng.random((rows, n)) < rng.random()
    elif kind == "causal":
        mask = np.tril(np.ones((rows, n), bool), k=n - rows)
    else:  # a prefix plus a few later keys
        mask = np.zeros((rows, n), bool)
        p = int(rng.integers(0, n))
        mask[:, :p] = True
        mask |= rng.random((rows, n)) < 0.1
    rp, ki = _csr(mask)
    kb, kl, trp, tail = cuda.split_runs(rp, ki)
    for r in range(rows):
        keys = list(range(kb[r], kb[r] + kl[r])) + list(tail[trp[r]:trp[r + 1]])
        assert keys == list(np.flatnonzero(mask[r]))
        if kl[r] < mask[r].sum():  # the run ends where the next key is not consecutive
            assert tail[trp[r]] != kb[r] + kl[r]


def test_mask_routing():
    """Causal rows: RANGE with row blocks; a short group (decode): segments; prefix + ancestors:
    HYBRID; scattered keys: CSR."""
    causal = np.tril(np.ones((300, 300), bool))
    kw = cuda.mask_launch_kwargs(*_csr(causal), 128, 128, "cpu")
    assert "blocks" in kw and "row_ptr" not in kw and int(kw["kv_len"].sum()) == int(causal.sum())
    dec = np.ones((2, 500), bool)
    assert "segments" in cuda.mask_launch_kwargs(*_csr(dec), 128, 128, "cpu")
    tree = np.zeros((64, 1100), bool)
    tree[:, :1024] = True
    tree[np.arange(64), 1024 + np.arange(64)] = True
    kw = cuda.mask_launch_kwargs(*_csr(tree), 128, 128, "cpu")
    assert "blocks" in kw and "row_ptr" in kw and int(kw["key_idx"].numel()) == 63  # row 0: 1024 extends its run
    scattered = np.zeros((8, 100), bool)
    scattered[:, ::3] = True
    kw = cuda.mask_launch_kwargs(*_csr(scattered), 128, 128, "cpu")
    assert "kv_base" not in kw and "row_ptr" in kw
    # other head sizes: ranges without the tensor-core tables
    kw = cuda.mask_launch_kwargs(*_csr(causal), 64, 64, "cpu")
    assert "blocks" not in kw and "segments" not in kw
