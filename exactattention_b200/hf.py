"""Hugging Face attention hook: ExactAttention as `attn_implementation="exact"`.

Mirrors the reference's speculative-decoding demo hook (scripts/spec_decode_demo.py:57-73
`exact_attention`, registered with transformers' AttentionInterface), backed by the CUDA path:
causal attention of the query block placed at the end of the key range (prefill, decode, or a
block of draft tokens), for every sequence and head. Query / key / value are rounded to bf16 bit
patterns as the reference does; the output is the certified bf16 result. Prefill-sized query
blocks run on the tensor-core prefill kernel, short ones on the decode kernel.

    from exactattention_b200 import hf
    hf.register()                                   # once
    model = AutoModelForCausalLM.from_config(cfg, attn_implementation="exact")
"""

from __future__ import annotations

import numpy as np

from . import cuda
from .formats import alpha_for


def _bits(t):
    import torch

    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16)


def exact_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """query (B, H, ql, D), key / value (B, Hkv, kl, D): row (b, h, i) attends the keys
    0 .. kl - ql + i of (b, h // (H / Hkv)). Returns ((B, ql, H, D) bf16, None). attention_mask is
    not read: the rows are causal with the queries at the end of the key range, as in the
    reference's hook (padding masks are not supported)."""
    import torch

    if dropout:
        raise ValueError("ExactAttention has no dropout")
    B, H, ql, D = query.shape
    Hkv, kl = key.shape[1], key.shape[2]
    g = H // Hkv
    dev = query.device
    q = _bits(query).reshape(B * H * ql, D)
    k = _bits(key).reshape(B * Hkv * kl, D)
    v = _bits(value).reshape(B * Hkv * kl, value.shape[-1])
    b = np.repeat(np.arange(B), H * ql)
    h = np.tile(np.repeat(np.arange(H), ql), B)
    i = np.tile(np.arange(ql), B * H)
    base = ((b * Hkv + h // g) * kl).astype(np.int64)
    lens = (kl - ql + 1 + i).astype(np.int64)
    alpha = alpha_for(float(scaling if scaling is not None else module.scaling))
    kw = dict(kv_base=torch.from_numpy(base).to(dev), kv_len=torch.from_numpy(lens).to(dev), max_row_keys=kl)
    if D == 128 and value.shape[-1] == 128:
        if g * ql <= 8:  # decode / a few draft tokens: one segment per (sequence, kv head)
            kw["segments"] = torch.from_numpy(cuda.row_segments(base)).to(dev)
            kw["splits"] = max(1, min(64, kl // 2048))
        else:
            kw["blocks"] = torch.from_numpy(cuda.row_blocks(base, lens)).to(dev)
    out, flags = cuda.launch(q, k, v, alpha, **kw)
    if int(flags.max().item()) == 2:
        from .formats import ExactAttentionDomainError

        raise ExactAttentionDomainError("non-finite attention input")
    o = out.view(torch.bfloat16).reshape(B, H, ql, value.shape[-1])
    return o.permute(0, 2, 1, 3).contiguous(), None


def register(name: str = "exact") -> None:
    """Registers the hook with transformers' AttentionInterface under `name`."""
    from transformers import AttentionInterface

    AttentionInterface.register(name, exact_attention)
