"""The allocation-free entry point, ea_attention_cuda_noalloc, against ea_launch_cuda.

It exists for callers that cannot allocate device memory while they run attention (during CUDA
graph capture, under an allocator that owns the GPU, in latency-bound loops): its scratch is a
fixed static device array. Two calls in a row must give the same bits as the allocating entry
point, so nothing from the previous call (which the shared array keeps) leaks into the next.
This file sorts last so that a run stopping at the first failure has run every other test.
"""

import numpy as np
import pytest

from gen import bf16

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)


def _case(seed, rows, n, kind):
    rng = np.random.default_rng(seed)
    Q, K, V = bf16(rng, (rows, 128), kind), bf16(rng, (n, 128), kind), bf16(rng, (n, 128), "wide")
    mask = rng.random((rows, n)) < 0.6
    counts = mask.sum(axis=1)
    rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    ki = np.concatenate([np.flatnonzero(m) for m in mask]).astype(np.int64)
    return Q, K, V, rp, ki


def test_no_alloc_matches_allocating_entry_point_twice(cuda_lib):
    import torch

    from exactattention_b200 import cuda
    from exactattention_b200.formats import default_alpha

    assert torch.cuda.is_available()
    dev = torch.device("cuda")
    alpha = default_alpha(128)
    # two different calls in a row, both with KV splits (the partials live in the scratch array)
    for seed, rows, n, kind, splits in ((1, 37, 400, "outlier", 4), (2, 64, 250, "normal", 3)):
        Q, K, V, rp, ki = _case(seed, rows, n, kind)
        args = (_t(Q, dev), _t(K, dev), _t(V, dev), alpha)
        kw = dict(row_ptr=_t(rp, dev), key_idx=_t(ki, dev), splits=splits)
        o_ref, f_ref = cuda.launch(*args, **kw)
        o_na, f_na = cuda.launch(*args, no_alloc=True, **kw)
        torch.cuda.synchronize()
        assert torch.equal(f_na, f_ref)
        assert torch.equal(o_na, o_ref)   # bit-exact: the spec has one correct output
        assert not f_na.any().item()


def test_no_alloc_rejects_oversize_calls(cuda_lib):
    import torch

    from exactattention_b200 import cuda
    from exactattention_b200.formats import default_alpha

    dev = torch.device("cuda")
    rows, n = 8192, 64
    Q = torch.zeros((rows, 128), dtype=torch.int16, device=dev)
    K = torch.zeros((n, 128), dtype=torch.int16, device=dev)
    kb = torch.zeros(rows, dtype=torch.int64, device=dev)
    kl = torch.full((rows,), n, dtype=torch.int64, device=dev)
    with pytest.raises(ValueError, match="maximum"):
        cuda.launch(Q, K, K, default_alpha(128), kv_base=kb, kv_len=kl, splits=16, no_alloc=True)
