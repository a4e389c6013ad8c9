"""CPU oracle for Inkling relative-position-bias attention (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference arm may import it.  The ``inkling_fa4`` package
never imports it, and the CUDA path has no CPU fallback.

It restates, in numpy float32, the algorithm of the reference oracle
``ref_rel_attn`` (src/inkling_fa4/reference.py:4-39 of KINGXD414/Inkling-FA4-Relative-Attention):

* per sequence ``b`` (reference.py:21-23) and per query head ``h`` (reference.py:25), with
  the GQA kv head ``h // (Hq // Hkv)`` (reference.py:20,26);
* dense scores ``S = (q_b[:,h] @ k_b[:,kh]^T) * scale`` in fp32 (reference.py:27);
* the bias distance ``d = (q_pos + (sq - sk)) - k_pos`` (reference.py:28-31), the bias
  ``rel[q, h, clamp(d, 0, R-1)]`` gathered and zeroed where ``not 0 <= d < R``
  (reference.py:32-34), added after scaling (reference.py:35);
* the causal mask ``q_pos >= k_pos`` and the window mask ``q_pos - k_pos <= window_left``
  on *local, un-offset* positions (reference.py:36-37);
* fp32 softmax over keys (fully masked rows give NaN, as torch does; reference.py:38) and
  ``P @ v`` (reference.py:39).

Parity pin: ``tests/golden/make_golden.py`` imports the real ``reference.py`` (only in the
container that has it) and writes its outputs to ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks this restatement against every fixture.

Extension (not in the reference): ``causal_align="bottom_right"`` shifts the mask diagonal by
``sk - sq`` and uses bias offset ``sk - sq`` (the flash-attention / vLLM convention for
chunked prefill and decode).  When ``sq == sk`` both alignments are identical, which is how
the bottom-right results are pinned transitively to the reference.

Rows are independent, so ``row_block`` evaluates the same per-row algorithm on blocks of query
rows to bound memory at long sequence lengths (the reference materialises the full
``[sq, sk]`` score matrix, which at 32k is ~4 GB per head).
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "rel_attn",
    "rel_attn_rows",
    "round_to_bf16",
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "alignment_offsets",
    "rel_attn_torch",
    "rel_attn_rows_torch",
]


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even) and return the raw uint16 bits."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounding_bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding_bias) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """Widen raw bfloat16 bits (uint16) to float32 exactly."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 value, returned as float32 (what ``tensor.to(bf16)`` stores)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def alignment_offsets(sq: int, sk: int, causal_align: str) -> tuple[int, int]:
    """Return ``(mask_shift, bias_shift)`` for one sequence.

    reference (reference.py:28-31,36-37): the mask compares local positions with no shift and
    the bias distance uses ``q_pos + (sq - sk) - k_pos``.
    bottom_right: both use ``q_pos + (sk - sq) - k_pos``.
    """
    if causal_align == "reference":
        return 0, sq - sk
    if causal_align == "bottom_right":
        return sk - sq, sk - sq
    raise ValueError(f"unknown causal_align {causal_align!r}")


def rel_attn_rows(q_rows, k_b, v_b, rel_rows, q_pos, sq, sk, scale, rel_extent,
                  causal=True, window_left=None, causal_align="reference", return_lse=False):
    """Attention for a block of query rows of one (sequence, head).

    ``q_rows`` [n, d], ``k_b``/``v_b`` [sk, d], ``rel_rows`` [n, >=rel_extent] (float32),
    ``q_pos`` [n] local query positions.  Returns float32 [n, d].
    Follows reference.py:27-39 row by row.
    """
    if sk == 0:  # softmax over an empty key axis: the reference's einsum yields zeros
        z = np.zeros((q_rows.shape[0], v_b.shape[1]), dtype=np.float32)
        return (z, np.full(q_rows.shape[0], -np.inf, np.float32)) if return_lse else z
    mask_shift, bias_shift = alignment_offsets(sq, sk, causal_align)
    scores = (q_rows @ k_b.T) * np.float32(scale)                       # reference.py:27
    qp = q_pos.reshape(-1, 1).astype(np.int64)
    kp = np.arange(sk, dtype=np.int64).reshape(1, -1)
    rel_dist = (qp + bias_shift) - kp                                    # reference.py:28-31
    in_range = (rel_dist >= 0) & (rel_dist < rel_extent)                 # reference.py:32
    idx = np.clip(rel_dist, 0, rel_extent - 1)
    bias = np.take_along_axis(rel_rows[:, :rel_extent], idx, axis=1)     # reference.py:33
    bias = np.where(in_range, bias, np.float32(0.0))                     # reference.py:34
    scores = scores + bias                                               # reference.py:35
    if causal:                                                           # reference.py:36
        scores = np.where(qp + mask_shift >= kp, scores, -np.inf)
    if window_left is not None:                                          # reference.py:37
        scores = np.where((qp + mask_shift - kp) <= window_left, scores, -np.inf)
    scores = scores.astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        m = np.max(scores, axis=1, keepdims=True)                        # reference.py:38
        e = np.exp(scores - m)
        ssum = np.sum(e, axis=1, keepdims=True)
        p = e / ssum
        # log-sum-exp of the same logits (an extension for LSE checks; -inf if all masked)
        lse = np.where(np.isfinite(m[:, 0]), m[:, 0] + np.log(ssum[:, 0]), -np.inf)
    o = (p.astype(np.float32) @ v_b).astype(np.float32)                 # reference.py:39
    return (o, lse.astype(np.float32)) if return_lse else o


def rel_attn(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, scale, rel_extent,
             causal=True, window_left=None, causal_align="reference", row_block=None,
             heads=None, out_bf16=False, return_lse=False):
    """numpy restatement of ``ref_rel_attn`` (reference.py:4-39).

    Args mirror the reference: q [Tq, Hq, d], k/v [Tk, Hkv, d], rel_logits [Tq, Hq, >=R]
    (any float dtype; converted to float32), cu_seqlens_* int arrays of length B+1.
    ``heads`` restricts the computation to a subset of query heads (others stay 0), used to
    time a bounded sample.  ``out_bf16`` rounds the result to bfloat16 values, which is what
    the reference stores when called with bf16 inputs (``out = zeros_like(q)``,
    reference.py:20,39).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    rel = np.asarray(rel_logits, dtype=np.float32)
    cu_q = np.asarray(cu_seqlens_q, dtype=np.int64)
    cu_k = np.asarray(cu_seqlens_k, dtype=np.int64)
    n_heads, kv_heads = q.shape[1], k.shape[1]
    g = n_heads // kv_heads
    out = np.zeros(q.shape, dtype=np.float32)
    lse_all = np.full((n_heads, q.shape[0]), -np.inf, dtype=np.float32)
    head_list = range(n_heads) if heads is None else heads
    for b in range(len(cu_q) - 1):                                       # reference.py:21
        qs, qe = int(cu_q[b]), int(cu_q[b + 1])
        ks, ke = int(cu_k[b]), int(cu_k[b + 1])
        sq, sk = qe - qs, ke - ks
        if sq == 0:
            continue
        blk = sq if not row_block else row_block
        for h in head_list:                                              # reference.py:25
            kh = h // g                                                  # reference.py:26
            k_b = np.ascontiguousarray(k[ks:ke, kh])
            v_b = np.ascontiguousarray(v[ks:ke, kh])
            for r0 in range(0, sq, blk):
                r1 = min(sq, r0 + blk)
                o, lse = rel_attn_rows(
                    q[qs + r0:qs + r1, h], k_b, v_b, rel[qs + r0:qs + r1, h],
                    np.arange(r0, r1), sq, sk, scale, rel_extent, causal, window_left,
                    causal_align, return_lse=True)
                out[qs + r0:qs + r1, h] = o
                lse_all[h, qs + r0:qs + r1] = lse
    if out_bf16:
        out = round_to_bf16(out)
    return (out, lse_all) if return_lse else out


def rel_attn_rows_torch(q_rows, k_b, v_b, rel_rows, q_pos, sq, sk, scale, rel_extent,
                        causal=True, window_left=None, causal_align="reference"):
    """``rel_attn_rows`` with torch CPU tensors (float32), which runs the elementwise steps on
    all intra-op threads.  Same steps, same citations (reference.py:27-39)."""
    import torch

    if sk == 0:
        return torch.zeros((q_rows.shape[0], v_b.shape[1]), dtype=torch.float32)
    mask_shift, bias_shift = alignment_offsets(sq, sk, causal_align)
    scores = (q_rows @ k_b.T) * scale
    qp = q_pos.view(-1, 1).to(torch.int64)
    kp = torch.arange(sk, dtype=torch.int64).view(1, -1)
    rel_dist = (qp + bias_shift) - kp
    in_range = (rel_dist >= 0) & (rel_dist < rel_extent)
    bias = torch.gather(rel_rows[:, :rel_extent], 1, rel_dist.clamp(0, rel_extent - 1))
    scores = scores + torch.where(in_range, bias, torch.zeros((), dtype=bias.dtype))
    if causal:
        scores = scores.masked_fill(~(qp + mask_shift >= kp), float("-inf"))
    if window_left is not None:
        scores = scores.masked_fill(~((qp + mask_shift - kp) <= window_left), float("-inf"))
    p = torch.softmax(scores, dim=-1)
    return p @ v_b


def rel_attn_torch(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, scale, rel_extent,
                   causal=True, window_left=None, causal_align="reference", row_block=None,
                   heads=None):
    """Torch-CPU twin of :func:`rel_attn` (float32 in, float32 out)."""
    import torch

    q, k, v = q.float(), k.float(), v.float()
    rel = rel_logits.float()
    n_heads, kv_heads = q.shape[1], k.shape[1]
    g = n_heads // kv_heads
    out = torch.zeros(q.shape, dtype=torch.float32)
    cu_q = [int(x) for x in cu_seqlens_q]
    cu_k = [int(x) for x in cu_seqlens_k]
    for b in range(len(cu_q) - 1):
        qs, qe, ks, ke = cu_q[b], cu_q[b + 1], cu_k[b], cu_k[b + 1]
        sq, sk = qe - qs, ke - ks
        if sq == 0:
            continue
        blk = sq if not row_block else row_block
        for h in (range(n_heads) if heads is None else heads):
            kh = h // g
            k_b = k[ks:ke, kh].contiguous()
            v_b = v[ks:ke, kh].contiguous()
            for r0 in range(0, sq, blk):
                r1 = min(sq, r0 + blk)
                out[qs + r0:qs + r1, h] = rel_attn_rows_torch(
                    q[qs + r0:qs + r1, h], k_b, v_b, rel[qs + r0:qs + r1, h],
                    torch.arange(r0, r1), sq, sk, scale, rel_extent, causal, window_left,
                    causal_align)
    return out


def rel_attn_grads_torch(q, k, v, rel_logits, dout, cu_seqlens_q, cu_seqlens_k, scale,
                         rel_extent, causal=True, window_left=None, causal_align="reference",
                         row_block=None):
    """Gradients (dq, dk, dv, drel) of ``sum(rel_attn_torch(...) * dout)`` by torch autograd
    (float32, CPU).  The reference has no backward; these are the gradients of its forward
    (reference.py:4-39), which autograd differentiates exactly.  Rows without a visible key
    (NaN in the reference's softmax) are given zero gradient, matching the kernels' zero
    output for such rows."""
    import torch

    leaves = [t.detach().float().clone().requires_grad_(True) for t in (q, k, v, rel_logits)]
    out = rel_attn_torch(*leaves, cu_seqlens_q, cu_seqlens_k, scale, rel_extent, causal=causal,
                         window_left=window_left, causal_align=causal_align, row_block=row_block)
    g = dout.detach().float().clone()
    g[torch.isnan(out)] = 0.0
    out = torch.nan_to_num(out, nan=0.0)
    (out * g).sum().backward()
    return tuple(torch.nan_to_num(t.grad, nan=0.0) for t in leaves)
