"""rel_logits producer: the step in front of the attention in the Inkling layer, fused into one
sm_100a kernel (``ifa4_rel_logits_launch``, include/inkling_fa4.h).

The reference repository has no code for this step, only its diagram
(outputs/architecture.md:51-64): ``RelLogitsProj`` (``einsum("thd,de->the", r, W)``, 16
features -> rel_extent) and the log-tau scaling ``tau = 1 + alpha * log(clamp((pos + 1) / nf,
1))`` (alpha = 0.1 there) both feeding ``rel_logits``.  This module reads the diagram as

    rel_logits[t, h, e] = tau(pos_t) * sum_j r[t, h, j] * W[j, e]

with ``W`` shared by all heads (``[16, R]``, the diagram's ``de``) or per head (``[H, 16, R]``),
fp32 arithmetic and one rounding to bf16.  ``alpha=0`` gives the plain projection.  The
output is the ``rel_logits`` tensor the attention entry points consume.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

D_REL = 16


@torch.no_grad()
def inkling_rel_logits(r, weight, cu_seqlens_q=None, cu_seqlens_k=None, *, alpha=0.0, nf=1.0,
                       out=None):
    """rel_logits ``[total_q, n_heads, rel_extent]`` (bf16) from the per-head relative features
    ``r [total_q, n_heads, 16]`` (bf16) and ``weight`` (``[16, R]`` or ``[n_heads, 16, R]``,
    bf16).

    Token positions for tau: ``t - cu_seqlens_q[b]`` inside sequence ``b`` (one sequence when
    ``cu_seqlens_q`` is None), shifted by ``len_k - len_q`` when ``cu_seqlens_k`` is given (the
    queries are the last ``len_q`` of ``len_k`` positions: chunked prefill, decode).  ``out``
    may be a wider ``[total_q, n_heads, >= R]`` buffer (columns ``[0, R)`` are written)."""
    if not isinstance(r, torch.Tensor) or not isinstance(weight, torch.Tensor):
        raise TypeError("rel_logits: r and weight must be torch.Tensors")
    if not r.is_cuda:
        raise ValueError("rel_logits: r must be a CUDA tensor (no CPU path exists)")
    if weight.device != r.device:
        raise ValueError(f"rel_logits: weight is on {weight.device}, r on {r.device}")
    if r.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("rel_logits: r and weight must be bfloat16")
    if r.dim() != 3 or r.shape[2] != D_REL:
        raise ValueError(f"rel_logits: r must be [total_q, n_heads, {D_REL}], got {tuple(r.shape)}")
    total_q, n_heads = r.shape[0], r.shape[1]
    if weight.dim() == 2:
        if weight.shape[0] != D_REL:
            raise ValueError(f"rel_logits: weight must be [{D_REL}, R] or [n_heads, {D_REL}, R]")
        w_sh, w_sj = 0, weight.stride(0)
    elif weight.dim() == 3:
        if weight.shape[0] != n_heads or weight.shape[1] != D_REL:
            raise ValueError(f"rel_logits: weight must be [{D_REL}, R] or [n_heads, {D_REL}, R]")
        w_sh, w_sj = weight.stride(0), weight.stride(1)
    else:
        raise ValueError(f"rel_logits: weight must be [{D_REL}, R] or [n_heads, {D_REL}, R]")
    rel_extent = weight.shape[-1]
    if (weight.stride(-1) != 1 or weight.data_ptr() % 16 or w_sh % 8 or w_sj % 8
            or w_sj <= 0):
        weight = weight.contiguous()
        w_sh, w_sj = (0, weight.stride(0)) if weight.dim() == 2 else weight.stride()[:2]
    if rel_extent % 8:
        raise ValueError(f"rel_logits: rel_extent {rel_extent} must be a multiple of 8")
    if not (math.isfinite(nf) and nf > 0) or not math.isfinite(alpha):
        raise ValueError("rel_logits: nf must be finite and > 0, alpha finite")
    if r.stride(-1) != 1 or any(s % 8 for s in r.stride()[:2]) or r.data_ptr() % 16:
        r = r.contiguous()
    batch = 1
    for nm, cu in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        if cu is None:
            continue
        if (not isinstance(cu, torch.Tensor) or cu.dtype != torch.int32 or cu.dim() != 1
                or cu.numel() < 2 or cu.device != r.device):
            raise ValueError(f"rel_logits: {nm} must be a 1-D int32 tensor [batch + 1] on r's "
                             "device")
    if cu_seqlens_k is not None and cu_seqlens_q is None:
        raise ValueError("rel_logits: cu_seqlens_k needs cu_seqlens_q")
    if cu_seqlens_q is not None:
        batch = cu_seqlens_q.numel() - 1
        if cu_seqlens_k is not None and cu_seqlens_k.numel() != batch + 1:
            raise ValueError("rel_logits: cu_seqlens_q and cu_seqlens_k differ in length")
        cu_seqlens_q = cu_seqlens_q.contiguous()
        cu_seqlens_k = None if cu_seqlens_k is None else cu_seqlens_k.contiguous()
    if out is None:
        out = torch.empty((total_q, n_heads, rel_extent), dtype=torch.bfloat16, device=r.device)
    elif (out.dtype != torch.bfloat16 or out.dim() != 3 or out.shape[0] != total_q
          or out.shape[1] != n_heads or out.shape[2] < rel_extent or out.device != r.device
          or out.stride(-1) != 1 or any(s % 8 for s in out.stride()[:2]) or out.data_ptr() % 16):
        raise ValueError("rel_logits: out must be bf16 [total_q, n_heads, >= R] on r's device with "
                         "unit last stride, strides multiple of 8 and 16-byte alignment")
    p = _lib.RelLogitsParams()
    p.r, p.weight, p.rel = r.data_ptr(), weight.data_ptr(), out.data_ptr()
    p.cu_seqlens_q = 0 if cu_seqlens_q is None else cu_seqlens_q.data_ptr()
    p.cu_seqlens_k = 0 if cu_seqlens_k is None else cu_seqlens_k.data_ptr()
    p.r_stride_t, p.r_stride_h = r.stride(0), r.stride(1)
    p.weight_stride_h, p.weight_stride_j = w_sh, w_sj
    p.rel_stride_t, p.rel_stride_h = out.stride(0), out.stride(1)
    p.total_q = total_q
    p.batch, p.n_heads, p.d_rel, p.rel_extent = batch, n_heads, D_REL, rel_extent
    p.dtype = _lib.IFA4_DTYPE_BF16
    p.alpha, p.nf = float(alpha), float(nf)
    with torch.cuda.device(r.device):
        stream = torch.cuda.current_stream(r.device).cuda_stream
        _lib.check(_lib.lib().ifa4_rel_logits_launch(ctypes.byref(p), ctypes.c_void_p(stream)))
    return out
