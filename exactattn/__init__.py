"""`exactattn`: the reference package's import name (src/exactattn/__init__.py:3-14), served by the
B200 library `exactattention_b200`, so that callers written against the reference run unchanged:

    import exactattn
    out = exactattn.attention(q_bits, k_bits, v_bits, alpha, mask=None, out="bf16")
    from exactattn.torch_impl import attention_torch
    from exactattn.cuda import attention_cuda     # the CUDA counterpart of exactattn.cpu.attention_cpu

`exactattn.cuda`, `exactattn.torch_impl` and `exactattn.formats` are the B200 package's modules
under those names. The reference's `trace_row` (exact intermediates for debugging) is not
provided: it belongs to the reference's pure-Python ground truth, not to the attention path.
"""

import sys as _sys

import exactattention_b200 as _ea
from exactattention_b200 import cuda, formats, torch_impl  # noqa: F401
from exactattention_b200 import (  # noqa: F401
    ExactAttentionDomainError,
    attention,
    attention_row,
    bf16_bits_to_float32,
    default_alpha,
    float_to_bf16_bits,
)

for _name in ("cuda", "formats", "torch_impl"):
    _sys.modules[f"{__name__}.{_name}"] = getattr(_ea, _name)

__all__ = [
    "ExactAttentionDomainError",
    "attention",
    "attention_row",
    "bf16_bits_to_float32",
    "default_alpha",
    "float_to_bf16_bits",
]
