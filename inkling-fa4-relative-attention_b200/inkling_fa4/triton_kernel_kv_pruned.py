"""KV-range-pruned prefill (drop-in name of src/inkling_fa4/triton_kernel_kv_pruned.py).

Every prefill launch in this package prunes: KV tiles entirely in the causal future or left
of the sliding window are never loaded (the tile range is computed per CTA before the first
TMA, csrc/ifa4_prefill_sm100.cu ``tile_info``).  This name is therefore an alias with the
reference's signature (triton_kernel_kv_pruned.py:210-226).
"""
from __future__ import annotations

from .triton_kernel import inkling_fa4_rel_attention_triton


def inkling_fa4_rel_attention_kv_pruned_triton(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k,
                                               max_seqlen_q, max_seqlen_k, rel_extent,
                                               causal=True, window_size=(-1, -1),
                                               n_heads=None, kv_heads=None, head_dim=128,
                                               arch=None, **kwargs):
    return inkling_fa4_rel_attention_triton(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k,
                                            max_seqlen_q, max_seqlen_k, rel_extent,
                                            causal=causal, window_size=window_size,
                                            n_heads=n_heads, kv_heads=kv_heads,
                                            head_dim=head_dim, arch=arch, **kwargs)


__all__ = ["inkling_fa4_rel_attention_kv_pruned_triton"]
