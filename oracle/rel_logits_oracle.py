"""CPU oracle for the rel_logits producer (TEST INFRASTRUCTURE ONLY).

Parity unpinned.  The reference repository (KINGXD414/Inkling-FA4-Relative-Attention) holds no
code for this step and no test of it: only its diagram, outputs/architecture.md:51-64, with

* ``RelLogitsProj``: ``einsum("thd,de->the", r, W)``, 16 features -> rel_extent;
* ``log_scaling_tau``: ``tau = 1 + alpha * log(clamp((pos + 1) / nf, 1))``, alpha = 0.1;
* both feeding ``rel_logits [total_q, H, rel_extent]``.

This module restates that reading in numpy float32 (products and sums in fp32, tau in fp32,
``rel = tau * proj``), which is also what ``ifa4_rel_logits_launch`` computes; it pins the
kernel to the formula, not to reference code, because none exists.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` may import it.
"""
from __future__ import annotations

import numpy as np

__all__ = ["token_positions", "log_tau", "rel_logits_proj"]


def token_positions(total_q, cu_seqlens_q=None, cu_seqlens_k=None):
    """Position of every token in its sequence: ``t - cu_q[b]``, plus ``len_k - len_q`` of its
    sequence when ``cu_seqlens_k`` is given (queries are the last ``len_q`` of ``len_k``
    positions).  Without ``cu_seqlens_q`` all tokens form one sequence."""
    t = np.arange(total_q, dtype=np.int64)
    if cu_seqlens_q is None:
        return t
    cu_q = np.asarray(cu_seqlens_q, dtype=np.int64)
    b = np.clip(np.searchsorted(cu_q, t, side="right") - 1, 0, len(cu_q) - 2)
    pos = t - cu_q[b]
    if cu_seqlens_k is not None:
        cu_k = np.asarray(cu_seqlens_k, dtype=np.int64)
        pos = pos + (cu_k[b + 1] - cu_k[b]) - (cu_q[b + 1] - cu_q[b])
    return pos


def log_tau(pos, alpha, nf):
    """``1 + alpha * log(max((pos + 1) / nf, 1))`` in float32, step by step."""
    ratio = (pos.astype(np.float32) + np.float32(1.0)) / np.float32(nf)
    lg = np.log(np.maximum(ratio, np.float32(1.0))).astype(np.float32)
    return (np.float32(1.0) + np.float32(alpha) * lg).astype(np.float32)


def rel_logits_proj(r, weight, cu_seqlens_q=None, cu_seqlens_k=None, alpha=0.0, nf=1.0):
    """float32 ``tau(pos_t) * einsum(r[t, h, :], W_h)`` for ``r [T, H, 16]`` and ``weight``
    ``[16, R]`` (shared) or ``[H, 16, R]`` (per head).  The kernel's bf16 output is this value
    rounded once to bf16."""
    r = np.asarray(r, dtype=np.float32)
    w = np.asarray(weight, dtype=np.float32)
    if w.ndim == 2:
        proj = np.einsum("thd,de->the", r, w, dtype=np.float32)
    else:
        proj = np.einsum("thd,hde->the", r, w, dtype=np.float32)
    pos = token_positions(r.shape[0], cu_seqlens_q, cu_seqlens_k)
    tau = log_tau(pos, alpha, nf) if alpha != 0.0 else np.ones(r.shape[0], np.float32)
    return (proj * tau[:, None, None]).astype(np.float32)
