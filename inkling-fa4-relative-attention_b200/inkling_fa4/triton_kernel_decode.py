"""Single-token decode entry point (drop-in name of src/inkling_fa4/triton_kernel_decode.py).

Split-KV HBM-streaming kernel plus combine kernel (csrc/ifa4_decode_sm100.cu) behind the C
ABI.  Semantics are those of the oracle ref_rel_attn (reference.py:4-39) with one query per
sequence; the reference's own decode kernel deviates from the oracle (1/sqrt(d) scale,
global-offset masks, triton_kernel_decode.py:57,73-75,88) and is not reproduced.
"""
from __future__ import annotations

from . import _ops


def inkling_fa4_rel_attention_decode_triton(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k,
                                            max_seqlen_q, max_seqlen_k, rel_extent,
                                            causal=True, window_size=(-1, -1),
                                            n_heads=None, kv_heads=None, head_dim=128,
                                            arch=None, *, softmax_scale=None,
                                            causal_align="reference", out=None,
                                            num_splits=0, chunk_len=0, workspace=None,
                                            return_lse=False, lse=None, block_table=None):
    """Decode: q [batch, n_heads, 128] (one query per sequence, cu_seqlens_q = 0..batch),
    k/v [total_k, kv_heads, 128], rel_logits [batch, n_heads, >=rel_extent].

    Arguments as in the reference (triton_kernel_decode.py:128-138).  ``max_seqlen_k`` sizes the
    split-KV plan (any value is safe: splits stride over key chunks).  Extensions:
    ``softmax_scale``, ``causal_align`` (use "bottom_right" for the usual decode semantics in
    which the query is the last position of its sequence; "reference" reproduces the oracle,
    whose query sees key 0 only), ``out``, ``num_splits``/``chunk_len`` (0 = automatic) and a
    reusable ``workspace`` (uint8 CUDA tensor; allocated per call when absent), and
    ``return_lse`` / ``lse`` and ``block_table`` (paged KV cache) as in the prefill entry
    point.
    """
    return _ops.decode(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                       max_seqlen_k, rel_extent, causal=causal, window_size=window_size,
                       n_heads=n_heads, kv_heads=kv_heads, head_dim=head_dim,
                       softmax_scale=softmax_scale, causal_align=causal_align, out=out,
                       num_splits=num_splits, chunk_len=chunk_len, workspace=workspace,
                       return_lse=return_lse, lse=lse, block_table=block_table)


__all__ = ["inkling_fa4_rel_attention_decode_triton"]
