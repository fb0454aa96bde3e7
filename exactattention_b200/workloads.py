"""The benchmark configurations, as seeded synthetic inputs (the reference's own numbers came from
captured Qwen3-0.6B activations, which are not available; these stand in with the same shapes and
the value distributions described for each config).

  c1  single head, d=64: q (2,64), k, v (100,64) ~ N(0,1) from default_rng(0), no mask
  c2  Qwen3-0.6B causal prefill: 16 q / 8 kv heads, d=128, 4096 tokens; q, k ~ N(0,1) times a
      per-(head, channel) scale 2^U(-2,2) with 2% of channels times U(8,16); v ~ N(0,1)
  c3  paged GQA decode: 64 sequences, contexts U[4096, 32768], page size 16, pages of all
      sequences permuted in one pool; c2's distributions; one query token per sequence
  c4  tree verification: 16 sequences, 8192-token prefix, a 64-node draft tree each (BFS,
      branching U{1..4}, depth <= 8); node rows attend prefix + their ancestors (self included)
  c5  long context: 4 sequences, 2^20 keys, one query token; q, k, v ~ N(0,1) with 1% of rows
      (independently per tensor) scaled by 32

Large tensors come from an integer-only generator (three splitmix64 hashes -> twelve 16-bit
uniforms -> Irwin-Hall normal -> exact RN to bf16), implemented identically here in numpy and
in CUDA (csrc/ea_synth.cu), so the CPU oracle and the GPU build the same bits independently.
Small structures (scales, context lengths, page tables, trees) come from numpy default_rng.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

from .formats import default_alpha, float_to_bf16_bits

D = 128
HQ, HKV = 16, 8
GROUP = HQ // HKV
T_Q, T_K, T_V = 1, 2, 3

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _sm_scalar(x: int) -> int:
    return int(_splitmix64(np.array([x & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64))[0])


def _rn_bf16(X: np.ndarray, E: np.ndarray) -> np.ndarray:
    """RN-even of X * 2^E (int64 X, normal range) to bf16 bits."""
    neg = X < 0
    a = np.abs(X).astype(np.uint64)
    L = np.zeros(a.shape, np.int64)
    nz = a != 0
    L[nz] = np.floor(np.log2(a[nz].astype(np.float64))).astype(np.int64) + 1
    # fix float log2 at powers of two
    L = np.where(nz & ((a >> np.clip(L - 1, 0, 63).astype(np.uint64)) == 0), L - 1, L)
    L = np.where(nz & ((a >> np.clip(L, 0, 63).astype(np.uint64)) != 0), L + 1, L)
    K = E + L - 1
    sh = np.clip(L - 8, 0, 63).astype(np.uint64)
    q = np.where(L <= 8, a << np.clip(8 - L, 0, 63).astype(np.uint64), a >> sh)
    rem = a & ((np.uint64(1) << sh) - np.uint64(1))
    half = np.where(sh > 0, np.uint64(1) << np.clip(sh.astype(np.int64) - 1, 0, 63).astype(np.uint64), np.uint64(0))
    up = (L > 8) & ((rem > half) | ((rem == half) & ((q & np.uint64(1)) == 1)))
    q = q + up.astype(np.uint64)
    carry = q == 256
    q = np.where(carry, np.uint64(128), q)
    K = K + carry
    bits = (np.where(neg, 0x8000, 0) | ((K + 127) << 7) | (q & np.uint64(0x7F)).astype(np.int64))
    return np.where(nz, bits, 0).astype(np.uint16)


@dataclass
class Scale:
    m: np.ndarray  # (H, D) int32 fp32 significands
    e: np.ndarray  # (H, D) int32 exponents

    @staticmethod
    def from_f32(x: np.ndarray) -> "Scale":
        f = np.asarray(x, np.float32)
        u = f.view(np.uint32).astype(np.int64)
        ex = (u >> 23) & 0xFF
        return Scale(((u & 0x7FFFFF) | 0x800000).astype(np.int32), (ex - 150).astype(np.int32))


def draw_scales(rng: np.random.Generator, heads: int, d: int = D) -> Scale:
    """2^U(-2, 2) per (head, channel); 2% of channels times U(8, 16)."""
    s = np.exp2(rng.uniform(-2, 2, size=(heads, d)))
    outl = rng.random((heads, d)) < 0.02
    s = np.where(outl, s * rng.uniform(8, 16, size=(heads, d)), s)
    return Scale.from_f32(s.astype(np.float32))


_host_gen = None


def _host_generator():
    """The C form of this generator (csrc/ea_synth_host.c, all host threads), or None when it is
    not built; both give the same bits."""
    global _host_gen
    if _host_gen is None:
        import ctypes
        import os

        p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libea_synth_host.so")
        if not os.path.exists(p):
            return None
        lib = ctypes.CDLL(p)
        P, I64 = ctypes.c_void_p, ctypes.c_int64
        lib.ea_synth_rows_host.argtypes = [P, ctypes.c_uint64, ctypes.c_uint64, I64, I64, I64, I64, I64, I64, I64,
                                           P, P, ctypes.c_int]
        lib.ea_synth_rows_host.restype = ctypes.c_int
        _host_gen = lib
    return _host_gen


def synth_rows(seed: int, tensor_id: int, shape, g: int, h: int, t0: int, t1: int, scale: Scale | None = None,
               heavy_permille: int = 0, chunk: int = 1 << 22, use_host_lib: bool = True) -> np.ndarray:
    """Rows [g, h, t0:t1, :] of the logical (G, H, T, D) tensor, as uint16 bf16 bits."""
    G, H, T, Dd = shape
    lib = _host_generator() if use_host_lib else None
    if lib is not None:
        out = np.empty((t1 - t0, Dd), np.uint16)
        sm = se = None
        if scale is not None:
            sm = np.ascontiguousarray(scale.m, np.int32)
            se = np.ascontiguousarray(scale.e, np.int32)
        rc = lib.ea_synth_rows_host(out.ctypes.data, seed, tensor_id, H, T, Dd, g, h, t0, t1,
                                    sm.ctypes.data if sm is not None else None,
                                    se.ctypes.data if se is not None else None, heavy_permille)
        if rc != 0:
            raise RuntimeError("ea_synth_rows_host failed")
        return out
    base = _sm_scalar((seed << 20) ^ tensor_id)
    hbase = _sm_scalar(base ^ 0x5555555555555555)
    out = np.empty((t1 - t0) * Dd, np.uint16)
    start = ((g * H + h) * T + t0) * Dd
    total = (t1 - t0) * Dd
    c_idx = np.arange(Dd, dtype=np.int64)
    for o in range(0, total, chunk):
        n = min(chunk, total - o)
        i = np.arange(start + o, start + o + n, dtype=np.uint64)
        b3 = np.uint64(base) + np.uint64(3) * i
        s = np.zeros(n, np.int64)
        for j in range(3):
            hh = _splitmix64(b3 + np.uint64(j))
            for k in range(4):
                s += ((hh >> np.uint64(16 * k)) & np.uint64(0xFFFF)).astype(np.int64)
        cv = s - 393210
        c = (i.astype(np.int64)) % Dd
        if scale is None:
            sm = np.full(n, 1 << 23, np.int64)
            se = np.full(n, -23, np.int64)
        else:
            sm = scale.m[h][c].astype(np.int64)
            se = scale.e[h][c].astype(np.int64)
        if heavy_permille:
            rowi = i // np.uint64(Dd)
            hv = (_splitmix64(np.uint64(hbase) + rowi) % np.uint64(1000)) < np.uint64(heavy_permille)
            se = se + 5 * hv
        out[o:o + n] = _rn_bf16(cv * sm, se - 16)
    del c_idx
    return out.reshape(t1 - t0, Dd)


# ---------------------------------------------------------------------------
# configurations
# ---------------------------------------------------------------------------

@dataclass
class Config:
    name: str
    seed: int
    batch: int
    q_tokens: int                       # query tokens per sequence (per head)
    kv_tokens: int                      # logical K/V tokens per sequence (T of the K tensor)
    q_scale: Scale | None = None
    k_scale: Scale | None = None
    heavy_permille: int = 0
    ctx: np.ndarray | None = None       # c3: context per sequence
    page_size: int = 0
    page_table: np.ndarray | None = None
    parents: list = field(default_factory=list)   # c4: per sequence parent arrays (64 nodes)
    depth: list = field(default_factory=list)
    prefix: int = 0

    @property
    def alpha(self) -> np.float32:
        return default_alpha(D)

    @property
    def rows(self) -> int:
        return self.batch * HQ * self.q_tokens

    def row_keys(self) -> np.ndarray:
        """keys attended by every row, in the canonical row order (b, h, token)."""
        if self.name == "c2":
            return np.tile(np.arange(1, self.q_tokens + 1, dtype=np.int64), HQ)
        if self.name == "c3":
            return np.repeat(self.ctx.astype(np.int64), HQ)
        if self.name == "c4":
            per = [np.array([self.prefix + d_ for d_ in dep], np.int64) for dep in self.depth]
            return np.concatenate([np.tile(p, HQ) for p in per])
        if self.name == "c5":
            return np.full(self.rows, self.kv_tokens, np.int64)
        raise ValueError(self.name)

    @property
    def pairs(self) -> int:
        return int(self.row_keys().sum())

    def ancestors(self, b: int, node: int) -> list[int]:
        path, x = [], node
        while x != -1:
            path.append(x)
            x = self.parents[b][x]
        return path[::-1]


def _tree(rng: np.random.Generator, nodes: int = 64, max_depth: int = 8):
    """BFS draft tree: each node below max_depth gets U{1..4} children until `nodes` exist."""
    parent, depth = [-1], [1]
    frontier = [0]
    while len(parent) < nodes:
        if not frontier:
            frontier = [i for i in range(len(parent)) if depth[i] < max_depth][:1]
        x = frontier.pop(0)
        if depth[x] >= max_depth:
            continue
        for _ in range(int(rng.integers(1, 5))):
            if len(parent) >= nodes:
                break
            parent.append(x)
            depth.append(depth[x] + 1)
            frontier.append(len(parent) - 1)
    return parent, depth


def config(name: str) -> Config:
    if name == "c2":
        rng = np.random.default_rng(2)
        return Config("c2", 2, 1, 4096, 4096, draw_scales(rng, HQ), draw_scales(rng, HKV))
    if name == "c3":
        rng = np.random.default_rng(3)
        qs, ks = draw_scales(rng, HQ), draw_scales(rng, HKV)
        B, ps = 64, 16
        ctx = rng.integers(4096, 32769, size=B)
        npages = (ctx + ps - 1) // ps
        max_pages = 32768 // ps
        perm = rng.permutation(int(npages.sum())).astype(np.int32)
        pt = np.full((B, max_pages), 0, np.int32)
        off = 0
        for b in range(B):
            pt[b, :npages[b]] = perm[off:off + npages[b]]
            off += int(npages[b])
        return Config("c3", 3, B, 1, 32768, qs, ks, ctx=ctx, page_size=ps, page_table=pt)
    if name == "c4":
        rng = np.random.default_rng(4)
        qs, ks = draw_scales(rng, HQ), draw_scales(rng, HKV)
        B, P, Nn = 16, 8192, 64
        par, dep = [], []
        for _ in range(B):
            p, d_ = _tree(rng, Nn)
            par.append(p)
            dep.append(d_)
        return Config("c4", 4, B, Nn, P + Nn, qs, ks, parents=par, depth=dep, prefix=P)
    if name == "c5":
        return Config("c5", 5, 4, 1, 1 << 20, heavy_permille=10)
    raise ValueError(name)


def c1():
    """(q, k, v, alpha) of config 1, the reference README's example (rng seed 0)."""
    rng = np.random.default_rng(0)
    q = float_to_bf16_bits(rng.standard_normal((2, 64)))
    k = float_to_bf16_bits(rng.standard_normal((100, 64)))
    v = float_to_bf16_bits(rng.standard_normal((100, 64)))
    return q, k, v, default_alpha(64)


# ---------------------------------------------------------------------------
# CPU side: per-(sequence, kv head) segments for the oracle
# ---------------------------------------------------------------------------

def segments(cfg: Config):
    """Yields (b, kvh, Q rows (r, D), K (n, D), V (n, D), row_ptr, key_idx, canonical row ids)."""
    H = HQ
    Tq = cfg.q_tokens
    for b in range(cfg.batch):
        for kvh in range(HKV):
            heads = [kvh * GROUP + i for i in range(GROUP)]
            qs = [synth_rows(cfg.seed, T_Q, (cfg.batch, HQ, Tq, D), b, h, 0, Tq, cfg.q_scale, cfg.heavy_permille)
                  for h in heads]
            Q = np.concatenate(qs)
            if cfg.name == "c3":
                n = int(cfg.ctx[b])
            else:
                n = cfg.kv_tokens
            K = synth_rows(cfg.seed, T_K, (cfg.batch, HKV, cfg.kv_tokens, D), b, kvh, 0, n, cfg.k_scale,
                           cfg.heavy_permille)
            V = synth_rows(cfg.seed, T_V, (cfg.batch, HKV, cfg.kv_tokens, D), b, kvh, 0, n, None, cfg.heavy_permille)
            if cfg.name == "c2":
                lens = np.arange(1, Tq + 1)
                one = [np.arange(x) for x in lens]
            elif cfg.name in ("c3", "c5"):
                one = [np.arange(n)]
            else:
                one = [np.concatenate([np.arange(cfg.prefix), cfg.prefix + np.array(cfg.ancestors(b, x))])
                       for x in range(Tq)]
            rows_keys = one * GROUP
            row_ptr = np.concatenate([[0], np.cumsum([len(x) for x in rows_keys])]).astype(np.int64)
            key_idx = np.concatenate(rows_keys).astype(np.int64)
            canon = np.concatenate([(b * H + h) * Tq + np.arange(Tq) for h in heads])
            yield b, kvh, Q, K, V, row_ptr, key_idx, canon


def reference_outputs(name: str, attention_fn, progress=None) -> np.ndarray:
    """Output bits of the whole config in canonical row order (b, h, token), from a CPU
    implementation with the reference CPU kernel's signature (q, k, v, alpha, row_ptr, key_idx)."""
    cfg = config(name)
    out = np.zeros((cfg.rows, D), np.uint16)
    for b, kvh, Q, K, V, rp, ki, canon in segments(cfg):
        res, _ = attention_fn(Q, K, V, cfg.alpha, rp, ki)
        out[canon] = res
        if progress:
            progress(b, kvh)
    return out


def reference_sha(name: str, attention_fn) -> str:
    return hashlib.sha256(reference_outputs(name, attention_fn).tobytes()).hexdigest()


# ---------------------------------------------------------------------------
# GPU side: the same tensors built on the device by csrc/ea_synth.cu
# ---------------------------------------------------------------------------

class _SynthSpec:
    pass


def _synth_struct():
    import ctypes

    class S(ctypes.Structure):
        _fields_ = [("seed", ctypes.c_uint64), ("tensor_id", ctypes.c_uint64),
                    ("G", ctypes.c_int64), ("H", ctypes.c_int64), ("T", ctypes.c_int64), ("D", ctypes.c_int64),
                    ("t0", ctypes.c_int64), ("T_full", ctypes.c_int64),
                    ("scale_m", ctypes.c_void_p), ("scale_e", ctypes.c_void_p), ("heavy_permille", ctypes.c_int),
                    ("lens", ctypes.c_void_p), ("page_table", ctypes.c_void_p), ("max_pages", ctypes.c_int),
                    ("page_size", ctypes.c_int)]
    return S


_SynthStruct = None


def synth_device(seed: int, tensor_id: int, shape, scale: Scale | None = None, heavy_permille: int = 0,
                 device="cuda", t0: int = 0, T_full: int = 0, lens=None, page_table=None, page_size: int = 0,
                 out=None):
    """Device tensor (int16 view of bf16 bits) equal to synth_rows of the same logical rows.
    With page_table/lens, writes the logical (G, H, T, D) tensor into paged storage `out`
    shaped (pages, H, page_size, D)."""
    import ctypes

    import torch

    from . import _lib

    global _SynthStruct
    if _SynthStruct is None:
        _SynthStruct = _synth_struct()
    lib = _lib.load()
    lib.ea_synth_fill.argtypes = [ctypes.c_void_p, ctypes.POINTER(_SynthStruct), ctypes.c_void_p]
    lib.ea_synth_fill.restype = ctypes.c_int
    G, H, T, Dd = shape
    dev = torch.device(device)
    if out is None:
        out = torch.empty((G, H, T, Dd), dtype=torch.int16, device=dev)
    keep = []
    s = _SynthStruct()
    s.seed, s.tensor_id, s.G, s.H, s.T, s.D, s.t0, s.T_full = seed, tensor_id, G, H, T, Dd, t0, T_full
    if scale is not None:
        sm = torch.from_numpy(scale.m.astype(np.int32)).to(dev)
        se = torch.from_numpy(scale.e.astype(np.int32)).to(dev)
        keep += [sm, se]
        s.scale_m, s.scale_e = sm.data_ptr(), se.data_ptr()
    s.heavy_permille = heavy_permille
    if lens is not None:
        ln = torch.as_tensor(np.asarray(lens, np.int32)).to(dev)
        keep.append(ln)
        s.lens = ln.data_ptr()
    if page_table is not None:
        pt = torch.as_tensor(np.asarray(page_table, np.int32)).to(dev)
        keep.append(pt)
        s.page_table, s.max_pages, s.page_size = pt.data_ptr(), pt.shape[1], page_size
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        rc = lib.ea_synth_fill(ctypes.c_void_p(out.data_ptr()), ctypes.byref(s), ctypes.c_void_p(stream))
        if rc != 0:
            raise RuntimeError(f"ea_synth_fill failed ({rc})")
        torch.cuda.current_stream(dev).synchronize()
    return out


def device_case(name: str, device="cuda", shard: int = 0, nshards: int = 1) -> dict:
    """Inputs of a config on the GPU plus the `cuda.launch` keyword arguments. Rows are in the
    canonical order (b, h, token). For c5, `shard`/`nshards` select a contiguous KV range of every
    (sequence, kv head): the rank's share of the multi-GPU run."""
    import torch

    cfg = config(name)
    dev = torch.device(device)
    B, Tq = cfg.batch, cfg.q_tokens
    q = synth_device(cfg.seed, T_Q, (B, HQ, Tq, D), cfg.q_scale, cfg.heavy_permille, dev).view(-1, D)
    kw: dict = {}
    if name == "c3":
        npages = int(cfg.page_table.max()) + 1
        kshape = (npages, HKV, cfg.page_size, D)
        k = torch.zeros(kshape, dtype=torch.int16, device=dev)
        v = torch.zeros(kshape, dtype=torch.int16, device=dev)
        for t_id, sc, buf in ((T_K, cfg.k_scale, k), (T_V, None, v)):
            synth_device(cfg.seed, t_id, (B, HKV, cfg.kv_tokens, D), sc, 0, dev, lens=cfg.ctx,
                         page_table=cfg.page_table, page_size=cfg.page_size, out=buf)
        kw = dict(page_table=torch.from_numpy(cfg.page_table).to(dev),
                  seq_lens=torch.from_numpy(cfg.ctx.astype(np.int32)).to(dev), page_size=cfg.page_size,
                  q_heads=HQ, kv_heads=HKV, max_row_keys=int(cfg.ctx.max()))
        return dict(cfg=cfg, q=q, k=k, v=v, kw=kw)
    T = cfg.kv_tokens
    t0, Tn = 0, T
    if name == "c5" and nshards > 1:
        t0, Tn = T * shard // nshards, T * (shard + 1) // nshards - T * shard // nshards
    k = synth_device(cfg.seed, T_K, (B, HKV, Tn, D), cfg.k_scale, cfg.heavy_permille, dev, t0=t0, T_full=T)
    v = synth_device(cfg.seed, T_V, (B, HKV, Tn, D), None, cfg.heavy_permille, dev, t0=t0, T_full=T)
    rows = cfg.rows
    r = np.arange(rows)
    b, h, tok = r // (HQ * Tq), (r // Tq) % HQ, r % Tq
    base = (b * HKV + h // GROUP) * Tn
    if name == "c2":
        from .cuda import row_blocks

        kw = dict(kv_base=torch.from_numpy(base.astype(np.int64)).to(dev),
                  kv_len=torch.from_numpy((tok + 1).astype(np.int64)).to(dev), max_row_keys=T,
                  blocks=torch.from_numpy(row_blocks(base, tok + 1)).to(dev))
    elif name == "c5":
        from .cuda import row_segments

        kw = dict(kv_base=torch.from_numpy(base.astype(np.int64)).to(dev),
                  kv_len=torch.from_numpy(np.full(rows, Tn, np.int64)).to(dev), max_row_keys=T,
                  segments=torch.from_numpy(row_segments(base)).to(dev), segment_width=GROUP)
    elif name == "c4":
        from .cuda import row_blocks

        tails = [np.array(cfg.ancestors(int(bb), int(tt)), np.int64) for bb, tt in zip(b, tok)]
        rp = np.concatenate([[0], np.cumsum([len(x) for x in tails])]).astype(np.int64)
        ki = np.concatenate([base[i] + cfg.prefix + tails[i] for i in range(rows)]).astype(np.int64)
        plen = np.full(rows, cfg.prefix, np.int64)
        kw = dict(kv_base=torch.from_numpy(base.astype(np.int64)).to(dev),
                  kv_len=torch.from_numpy(plen).to(dev),
                  row_ptr=torch.from_numpy(rp).to(dev), key_idx=torch.from_numpy(ki).to(dev),
                  max_row_keys=cfg.prefix + 8, blocks=torch.from_numpy(row_blocks(base, plen)).to(dev))
    return dict(cfg=cfg, q=q, k=k.view(-1, D), v=v.view(-1, D), kw=kw)
