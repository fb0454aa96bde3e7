"""KV-cache write path (ea_kv_append_cuda): tokens appended in steps into paged storage give the
cache, the per-key summary and the attention bits of writing everything at once (B200 only)."""

import numpy as np
import pytest

from gen import bf16

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)


def k_summary(rows: np.ndarray) -> np.ndarray:
    """numpy restatement of the per-key summary: max |k| bits | min nonzero |k| bits << 16."""
    mag = rows.astype(np.uint32) & 0x7FFF
    mx = mag.max(axis=-1)
    mn = np.where(mag == 0, 0xFFFF, mag).min(axis=-1)
    return (mx | (mn << 16)).astype(np.uint32)


def test_append_in_steps_equals_one_write_and_decodes_the_same():
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    rng = np.random.default_rng(808)
    B, hq, hkv, ps, d = 3, 4, 2, 16, 128
    final = rng.integers(100, 600, size=B)
    npg = (final + ps - 1) // ps
    perm = rng.permutation(int(npg.sum())).astype(np.int32)
    pt = np.zeros((B, int(npg.max())), np.int32)
    off = 0
    for b in range(B):
        pt[b, :npg[b]] = perm[off:off + npg[b]]
        off += int(npg[b])
    T = int(final.max())
    Kall = bf16(rng, (B, hkv, T, d), "outlier")
    Vall = bf16(rng, (B, hkv, T, d))
    Kall[1, 0, 5, 7] = 0x7FC0  # a NaN key row: the summary flags it
    dev = torch.device("cuda")
    shape = (int(npg.sum()), hkv, ps, d)
    kc = torch.zeros(shape, dtype=torch.int16, device=dev)
    vc = torch.zeros(shape, dtype=torch.int16, device=dev)
    meta = torch.zeros(shape[:3], dtype=torch.int32, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    ptd = _t(pt, dev)
    # steps of 37 tokens (a prefill chunk), then single tokens (decode); every sequence grows
    # by the same amount per step, so sequences stop at min(final) and the rest is appended after
    step_lens = [37, 37, 1, 1, 1, 50]
    cur = 0
    for n in step_lens:
        if cur + n > int(final.min()):
            break
        cuda.kv_append(kc, vc, ptd, lens, _t(np.ascontiguousarray(Kall[:, :, cur:cur + n]), dev),
                       _t(np.ascontiguousarray(Vall[:, :, cur:cur + n]), dev), k_meta=meta)
        cur += n
    for b in range(B):  # the rest per sequence (batch of one)
        n = int(final[b]) - cur
        if n:
            cuda.kv_append(kc, vc, ptd[b:b + 1], lens[b:b + 1], _t(np.ascontiguousarray(Kall[b:b + 1, :, cur:]), dev)[:, :, :n],
                           _t(np.ascontiguousarray(Vall[b:b + 1, :, cur:]), dev)[:, :, :n], k_meta=meta)
    torch.cuda.synchronize()
    assert lens.cpu().numpy().tolist() == final.tolist()
    # the expected cache, written directly
    Kc = np.zeros(shape, np.uint16)
    Vc = np.zeros(shape, np.uint16)
    Mc = np.zeros(shape[:3], np.uint32)
    for b in range(B):
        for j in range(int(final[b])):
            p = pt[b, j // ps]
            Kc[p, :, j % ps] = Kall[b, :, j]
            Vc[p, :, j % ps] = Vall[b, :, j]
            Mc[p, :, j % ps] = k_summary(Kall[b, :, j])
    assert np.array_equal(kc.cpu().numpy().view(np.uint16), Kc)
    assert np.array_equal(vc.cpu().numpy().view(np.uint16), Vc)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), Mc)
    assert (Mc[pt[1, 0], 0, 5] & 0xFFFF) >= 0x7F80
    # attention over the appended cache = over the directly written one
    Q = bf16(rng, (B * hq, d), "outlier")
    alpha = ea.default_alpha(d)
    kw = dict(page_table=ptd, seq_lens=lens, page_size=ps, q_heads=hq, kv_heads=hkv, splits=2)
    o1, f1 = cuda.launch(_t(Q, dev), kc, vc, alpha, **kw)
    o2, f2 = cuda.launch(_t(Q, dev), _t(Kc, dev), _t(Vc, dev), alpha, **kw)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(f1, f2)
    assert f1.cpu().numpy()[4:8].tolist() == [2, 2, 0, 0]  # sequence 1, kv head 0 sees the NaN
