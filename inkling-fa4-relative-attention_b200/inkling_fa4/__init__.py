"""inkling_fa4 — B200 (sm_100a) relative-position-bias flash attention.

Drop-in for the reference package's call surface (src/inkling_fa4/__init__.py:1-10):
``inkling_fa4_rel_attention_triton`` (prefill / varlen / chunked / sliding window),
``inkling_fa4_rel_attention_decode_triton`` (split-KV decode), ``ref_rel_attn`` (dense PyTorch
statement for tests) and ``autotune_configs``; beyond the reference, the backward
(``inkling_fa4_rel_attention_backward``), a differentiable ``inkling_fa4_rel_attention`` and the
fused ``rel_logits`` producer (``inkling_rel_logits``).  The kernels are hand-written CUDA for sm_100a
behind the C ABI of include/inkling_fa4.h; there is no Triton and no CPU fallback.
"""
from .triton_kernel import inkling_fa4_rel_attention_triton
from .reference import ref_rel_attn
from . import autotune_configs
from .triton_kernel_decode import inkling_fa4_rel_attention_decode_triton
from .backward import inkling_fa4_rel_attention, inkling_fa4_rel_attention_backward
from .rel_logits import inkling_rel_logits

__all__ = [
    "inkling_fa4_rel_attention_triton",
    "inkling_fa4_rel_attention_decode_triton",
    "ref_rel_attn",
    "autotune_configs",
    "inkling_fa4_rel_attention",
    "inkling_fa4_rel_attention_backward",
    "inkling_rel_logits",
]
