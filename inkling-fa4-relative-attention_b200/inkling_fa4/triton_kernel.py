"""Prefill / varlen / chunked / sliding-window entry point (drop-in name).

The module keeps the reference's name (src/inkling_fa4/triton_kernel.py) so existing imports
keep working; it contains no Triton.  The call goes through the C ABI to the sm_100a
tcgen05/TMA kernel in csrc/ifa4_prefill_sm100.cu.
"""
from __future__ import annotations

from . import _ops


def inkling_fa4_rel_attention_triton(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k,
                                     max_seqlen_q, max_seqlen_k, rel_extent,
                                     causal=True, window_size=(-1, -1),
                                     n_heads=None, kv_heads=None, head_dim=128,
                                     arch=None, *, softmax_scale=None,
                                     causal_align="reference", out=None, return_lse=False,
                                     lse=None, block_table=None):
    """Relative-position-bias flash attention over packed variable-length sequences.

    Same arguments and meaning as the reference (triton_kernel.py:84-106):
    q [total_q, n_heads, 128], k/v [total_k, kv_heads, 128], rel_logits
    [total_q, n_heads, >=rel_extent] (bf16; token stride 0 allowed), cu_seqlens_q/k int32
    [batch+1] on the device.  ``window_size[0]`` is the left window (-1: none);
    ``window_size[1]`` is ignored, as in the reference.  ``max_seqlen_q`` sizes the grid
    (any value is safe: CTAs stride over query tiles); ``max_seqlen_k`` is unused; ``arch`` is
    accepted and ignored (only sm_100a kernels exist).

    Extensions (keyword-only): ``softmax_scale`` (default 1/head_dim, the scale the reference
    kernel hard-codes, triton_kernel.py:55), ``causal_align`` ("reference": mask diagonal at
    local positions and bias offset sq - sk, reference.py:28-37; "bottom_right": both offset by
    sk - sq, the flash-attention convention for chunked prefill and decode), ``out``.

    Returns ``out`` [total_q, n_heads, 128] bf16.  Rows with no visible key are 0.  With
    ``return_lse=True`` (or an ``lse`` buffer) also returns the fp32 natural-log log-sum-exp of
    each row's scaled+biased logits, [n_heads, total_q] (-inf for rows with no visible key), for
    merging attention computed over separate key ranges.

    ``block_table`` (int32 [batch, max_pages]) switches k / v to a paged KV cache
    [num_pages, page_size, kv_heads, 128] (page_size a power of two >= 16): key j of sequence b
    is slot j % page_size of page block_table[b, j // page_size]; cu_seqlens_k still gives the
    key counts.  Cache slots past a sequence's last key are never used.
    """
    return _ops.prefill(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                        max_seqlen_k, rel_extent, causal=causal, window_size=window_size,
                        n_heads=n_heads, kv_heads=kv_heads, head_dim=head_dim,
                        softmax_scale=softmax_scale, causal_align=causal_align, out=out,
                        return_lse=return_lse, lse=lse, block_table=block_table)


__all__ = ["inkling_fa4_rel_attention_triton"]
