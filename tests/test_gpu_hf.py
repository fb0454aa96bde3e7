"""The Hugging Face hook (attn_implementation="exact") on the CUDA path (B200 only)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ql,kl", [(1, 700), (5, 300), (200, 200)])
def test_hook_rows_equal_the_oracle(ql, kl):
    import torch

    from exactattention_b200 import hf
    from exactattention_b200.formats import alpha_for
    from oracle import exact

    torch.manual_seed(ql)
    B, H, Hkv, D = 2, 4, 2, 128
    dev = torch.device("cuda")
    q = torch.randn(B, H, ql, D, device=dev)
    k = torch.randn(B, Hkv, kl, D, device=dev)
    v = torch.randn(B, Hkv, kl, D, device=dev)

    class M:
        scaling = D ** -0.5

    o, w = hf.exact_attention(M(), q, k, v, None, scaling=M.scaling)
    torch.cuda.synchronize()
    assert w is None and o.shape == (B, ql, H, D) and o.dtype == torch.bfloat16
    bits = lambda t: t.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    qb, kb, vb, ob = bits(q), bits(k), bits(v), bits(o)
    alpha = alpha_for(M.scaling)
    for b, h, i in ((0, 0, 0), (1, 3, ql - 1), (0, 2, ql // 2)):
        n = kl - ql + 1 + i
        ref = exact.attention_row(qb[b, h, i], kb[b, h // 2, :n], vb[b, h // 2, :n], alpha)
        assert np.array_equal(ob[b, i, h], ref), (b, h, i)


def test_tiny_qwen3_runs_with_the_hook():
    import torch
    from transformers import AutoModelForCausalLM, Qwen3Config

    from exactattention_b200 import hf

    hf.register()
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=512)
    torch.manual_seed(0)
    model = AutoModelForCausalLM.from_config(cfg, attn_implementation="exact").to("cuda", torch.bfloat16).eval()
    ids = torch.randint(0, 512, (1, 40), device="cuda")
    with torch.no_grad():
        a = model(ids).logits
        b = model(ids).logits
        gen = model.generate(ids, max_new_tokens=4, do_sample=False)
    assert torch.isfinite(a.float()).all() and torch.equal(a, b)
    assert gen.shape == (1, 44)
