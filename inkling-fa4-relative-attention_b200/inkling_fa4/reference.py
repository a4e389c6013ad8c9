"""``ref_rel_attn``: dense PyTorch statement of the oracle (drop-in for
src/inkling_fa4/reference.py:4-39), kept because the reference package exports it for tests.

It is a test utility: no kernel entry point calls it and it is not a fallback.  It follows the
reference line by line (per sequence and head: scaled scores, bias gather with zero outside
[0, rel_extent), causal/window masks on local positions, fp32 softmax, P V), and adds the
``causal_align`` keyword of the kernels ("bottom_right" shifts mask and bias by sk - sq).
"""
from __future__ import annotations

import torch


def ref_rel_attn(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, scale, rel_extent,
                 causal=True, window_left=None, causal_align="reference"):
    n_heads, kv_heads = q.shape[1], k.shape[1]
    batch = cu_seqlens_q.shape[0] - 1
    g = n_heads // kv_heads
    out = torch.zeros_like(q)
    for b in range(batch):
        qs, qe = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        ks, ke = int(cu_seqlens_k[b]), int(cu_seqlens_k[b + 1])
        sq, sk = qe - qs, ke - ks
        if causal_align == "reference":
            mask_shift, bias_shift = 0, sq - sk
        elif causal_align == "bottom_right":
            mask_shift, bias_shift = sk - sq, sk - sq
        else:
            raise ValueError(causal_align)
        q_b, rl_b = q[qs:qe].float(), rel_logits[qs:qe].float()
        q_pos = torch.arange(sq, device=q.device).view(-1, 1)
        k_pos = torch.arange(sk, device=q.device).view(1, -1)
        dist = (q_pos + bias_shift) - k_pos
        in_range = (dist >= 0) & (dist < rel_extent)
        idx = dist.clamp(0, rel_extent - 1)
        for h in range(n_heads):
            kh = h // g
            scores = (q_b[:, h] @ k[ks:ke, kh].float().T) * scale
            bias = torch.gather(rl_b[:, h, :rel_extent], 1, idx)
            bias[~in_range] = 0.0
            scores = scores + bias
            if causal:
                scores[~(q_pos + mask_shift >= k_pos)] = -float("inf")
            if window_left is not None:
                scores[~((q_pos + mask_shift - k_pos) <= window_left)] = -float("inf")
            p = torch.softmax(scores.to(torch.float32), dim=-1)
            out[qs:qe, h] = (p @ v[ks:ke, kh].float()).to(out.dtype)
    return out
