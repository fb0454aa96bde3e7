"""The device entry point inside CUDA graphs (a batched serving step): captured once after the
workspace is reserved, replayed with new inputs written into the same buffers, every replay gives
the bits of a plain launch (B200 only)."""

import numpy as np
import pytest

from gen import bf16

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).to(dev)


def _paged(rng, B=3, hq=4, hkv=2, ps=16):
    ctx = rng.integers(200, 900, size=B)
    npg = (ctx + ps - 1) // ps
    perm = rng.permutation(int(npg.sum())).astype(np.int32)
    pt = np.zeros((B, int(npg.max())), np.int32)
    off = 0
    for b in range(B):
        pt[b, :npg[b]] = perm[off:off + npg[b]]
        off += int(npg[b])
    Kc = bf16(rng, (int(npg.sum()), hkv, ps, 128), "outlier")
    Vc = bf16(rng, (int(npg.sum()), hkv, ps, 128))
    return Kc, Vc, pt, ctx, B * hq


@pytest.mark.parametrize("path", ["decode", "prefill", "csr"])
def test_graph_replay_matches_launch(path):
    import torch

    import exactattention_b200 as ea
    from exactattention_b200 import cuda

    rng = np.random.default_rng({"decode": 1, "prefill": 2, "csr": 3}[path])
    dev = torch.device("cuda")
    alpha = ea.default_alpha(128)
    if path == "decode":
        Kc, Vc, pt, ctx, rows = _paged(rng)
        k, v = _t(Kc, dev), _t(Vc, dev)
        kw = dict(page_table=_t(pt, dev), seq_lens=_t(ctx.astype(np.int32), dev), page_size=16, q_heads=4, kv_heads=2,
                  max_row_keys=int(ctx.max()), splits=3)
    elif path == "prefill":
        S, heads = 300, 2
        rows = heads * S
        k, v = _t(bf16(rng, (S, 128)), dev), _t(bf16(rng, (S, 128)), dev)
        kb = np.zeros(rows, np.int64)
        kl = np.tile(np.arange(1, S + 1, dtype=np.int64), heads)
        kw = dict(kv_base=_t(kb, dev), kv_len=_t(kl, dev), max_row_keys=S, blocks=_t(cuda.row_blocks(kb, kl), dev))
    else:
        n, rows = 500, 40
        k, v = _t(bf16(rng, (n, 64)), dev), _t(bf16(rng, (n, 64)), dev)
        lens = rng.integers(1, n, size=rows)
        rp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        ki = np.concatenate([rng.choice(n, size=int(m), replace=False) for m in lens]).astype(np.int64)
        kw = dict(row_ptr=_t(rp, dev), key_idx=_t(ki, dev), max_row_keys=int(lens.max()), splits=2)
    d = k.shape[-1]
    q = _t(bf16(rng, (rows, d), "outlier"), dev)
    out = torch.empty((rows, v.shape[-1]), dtype=torch.int16, device=dev)
    flags = torch.empty(rows, dtype=torch.uint8, device=dev)
    cuda.reserve_workspace(rows, kw.get("splits", 1), v.shape[-1])
    cuda.launch(q, k, v, alpha, out_tensor=out, flags=flags, **kw)  # warm-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cuda.launch(q, k, v, alpha, out_tensor=out, flags=flags, **kw)
    for trial in range(3):
        q.copy_(_t(bf16(rng, (rows, d), "outlier"), dev))  # a new step's queries, same buffer
        g.replay()
        ref_o, ref_f = cuda.launch(q.clone(), k, v, alpha, **kw)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_o) and torch.equal(flags, ref_f), trial
        assert not flags.any().item()
    del g
