"""The allocation-free entry point, ea_attention_cuda_noalloc, against ea_launch_cuda and the oracle.

It exists for callers that cannot allocate device memory while they run attention: a serving
process whose memory pool owns the whole GPU, or a latency-bound loop that cannot stall on a first
cudaMalloc. Its scratch is a fixed static device array. Two calls in a row must give the same bits
as the allocating entry point (and the oracle), so nothing from the previous call, which the shared
array keeps, leaks into the next; a warmed call must leave the device's free memory unchanged; and
the entry must work as the first call of a fresh process. This file sorts last so that a run
stopping at the first failure has run every other test.
"""

import os
import subprocess
import sys

import numpy as np
import pytest

from gen import bf16

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


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
    return Q, K, V, rp, ki, mask


CASES = ((1, 37, 400, "outlier", 4), (2, 64, 250, "normal", 3))


def test_no_alloc_matches_allocating_entry_point_twice(cuda_lib):
    import torch

    from exactattention_b200 import cuda
    from exactattention_b200.formats import default_alpha
    from oracle import exact

    assert torch.cuda.is_available()
    dev = torch.device("cuda")
    alpha = default_alpha(128)
    # two different calls in a row, both with KV splits (the partials live in the scratch array)
    for seed, rows, n, kind, splits in CASES:
        Q, K, V, rp, ki, mask = _case(seed, rows, n, kind)
        args = (_t(Q, dev), _t(K, dev), _t(V, dev), alpha)
        kw = dict(row_ptr=_t(rp, dev), key_idx=_t(ki, dev), splits=splits)
        o_ref, f_ref = cuda.launch(*args, **kw)
        o_na, f_na = cuda.launch(*args, no_alloc=True, **kw)
        torch.cuda.synchronize()
        assert torch.equal(f_na, f_ref)
        assert torch.equal(o_na, o_ref)   # bit-exact: the spec has one correct output
        assert not f_na.any().item()
        ora = exact.attention(Q, K, V, alpha, mask=mask)
        assert np.array_equal(o_na.cpu().numpy().view(np.uint16), ora)


def test_no_alloc_call_leaves_device_memory_unchanged(cuda_lib):
    """After a warm-up call (which looks up the array's address), a call changes neither the
    device's free memory nor torch's allocator."""
    import torch

    from exactattention_b200 import cuda
    from exactattention_b200.formats import default_alpha

    dev = torch.device("cuda")
    Q, K, V, rp, ki, _ = _case(3, 48, 300, "normal")
    args = (_t(Q, dev), _t(K, dev), _t(V, dev), default_alpha(128))
    kw = dict(row_ptr=_t(rp, dev), key_idx=_t(ki, dev), splits=4, max_row_keys=int(np.diff(rp).max()))
    out = torch.empty((48, 128), dtype=torch.int16, device=dev)
    flags = torch.empty(48, dtype=torch.uint8, device=dev)
    cuda.launch(*args, out_tensor=out, flags=flags, no_alloc=True, **kw)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    cuda.launch(*args, out_tensor=out, flags=flags, no_alloc=True, **kw)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0 and torch.cuda.memory_allocated() == alloc0


FRESH = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, {root!r}); sys.path.insert(0, {here!r})
from test_zz_no_alloc import _case, _t, CASES
from exactattention_b200 import cuda
from exactattention_b200.formats import default_alpha
from oracle import exact
dev = torch.device("cuda")
alpha = default_alpha(128)
outs = []
for seed, rows, n, kind, splits in CASES:  # the no-alloc entry first, before any other call
    Q, K, V, rp, ki, mask = _case(seed, rows, n, kind)
    o, f = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, row_ptr=_t(rp, dev), key_idx=_t(ki, dev),
                       splits=splits, no_alloc=True)
    outs.append((o.cpu().numpy().view(np.uint16), f.cpu().numpy(), Q, K, V, rp, ki, mask, splits))
for o, f, Q, K, V, rp, ki, mask, splits in outs:
    assert not f.any()
    assert np.array_equal(o, exact.attention(Q, K, V, alpha, mask=mask))
    o2, _ = cuda.launch(_t(Q, dev), _t(K, dev), _t(V, dev), alpha, row_ptr=_t(rp, dev), key_idx=_t(ki, dev),
                        splits=splits)
    assert np.array_equal(o, o2.cpu().numpy().view(np.uint16))
print("fresh ok")
"""


def test_no_alloc_first_call_in_a_fresh_process(cuda_lib):
    root = os.path.abspath(os.path.join(HERE, ".."))
    r = subprocess.run([sys.executable, "-c", FRESH.format(root=root, here=HERE)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "fresh ok" in r.stdout, r.stdout + r.stderr


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
    # rows x splits past the array in any arithmetic: refused before any size product is formed
    with pytest.raises(ValueError, match="maximum"):
        cuda.launch(Q, K, K, default_alpha(128), kv_base=kb, kv_len=kl, splits=65535, no_alloc=True)
