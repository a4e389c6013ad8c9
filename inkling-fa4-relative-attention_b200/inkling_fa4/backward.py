"""Backward pass and a differentiable entry point (not in the reference, which has forward
kernels only).  The gradients are those of the reference forward (src/inkling_fa4/reference.py
:4-39): dq, dk, dv and the gradient of rel_logits, computed by the sm_100a kernels behind
``ifa4_backward_launch`` (C ABI, include/inkling_fa4.h)."""
from __future__ import annotations

import ctypes

import torch

from . import _lib, _ops


@torch.no_grad()
def inkling_fa4_rel_attention_backward(dout, q, k, v, rel_logits, out, lse, cu_seqlens_q,
                                       cu_seqlens_k, max_seqlen_q, max_seqlen_k, rel_extent,
                                       causal=True, window_size=(-1, -1), n_heads=None,
                                       kv_heads=None, head_dim=128, softmax_scale=None,
                                       causal_align="reference", dq=None, dk=None, dv=None,
                                       drel=None, workspace=None):
    """Gradients (dq, dk, dv, drel) of the prefill given ``dout`` and the forward's ``out`` and
    ``lse`` ([n_heads, total_q] fp32, from ``return_lse=True``).  dq / dk / dv are bf16 like
    q / k / v; drel has rel_logits' shape (bf16), zero outside the band of distances
    [0, rel_extent) that reach a visible key."""
    q, k, v, rel, out_, n_heads, kv_heads, rel_extent, window_left, scale = _ops._prepare(
        "backward", q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, rel_extent, causal,
        window_size, n_heads, kv_heads, head_dim, softmax_scale, causal_align, out)
    for nm, t in (("dout", dout), ("lse", lse)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.device != q.device:
            raise ValueError(f"backward: {nm} must be a CUDA tensor on q's device")
    if dout.shape != q.shape or dout.dtype != q.dtype:
        raise ValueError("backward: dout must match q in shape and dtype")
    if lse.dtype != torch.float32 or lse.shape != (n_heads, q.shape[0]):
        raise ValueError("backward: lse must be float32 [n_heads, total_q]")
    dout = _ops._tma_ready(dout)
    out_ = _ops._tma_ready(out_)
    dq = torch.empty_like(q, memory_format=torch.contiguous_format) if dq is None else dq
    dk = torch.empty_like(k, memory_format=torch.contiguous_format) if dk is None else dk
    dv = torch.empty_like(v, memory_format=torch.contiguous_format) if dv is None else dv
    for nm, t, ref in (("dq", dq, q), ("dk", dk, k), ("dv", dv, v)):
        if t.shape != ref.shape or t.dtype != ref.dtype or t.device != ref.device:
            raise ValueError(f"backward: {nm} must match its input in shape, dtype and device")
        if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16:
            raise ValueError(f"backward: {nm} needs unit last stride, strides multiple of 8, "
                             "16-B alignment")
    if drel is None:
        width = rel_logits.shape[2]
        drel = (torch.zeros if width > rel_extent else torch.empty)(
            rel_logits.shape, dtype=rel_logits.dtype, device=q.device)
    elif drel.shape != rel_logits.shape or drel.dtype != rel_logits.dtype or drel.stride(-1) != 1:
        raise ValueError("backward: drel must match rel_logits with a unit last stride")
    p = _lib.BackwardParams()
    p.q, p.k, p.v, p.rel = q.data_ptr(), k.data_ptr(), v.data_ptr(), rel.data_ptr()
    p.out, p.dout, p.lse = out_.data_ptr(), dout.data_ptr(), lse.data_ptr()
    p.dq, p.dk, p.dv, p.drel = dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), drel.data_ptr()
    p.cu_seqlens_q, p.cu_seqlens_k = cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr()
    for nm, t in (("q", q), ("k", k), ("v", v), ("rel", rel), ("out", out_), ("dout", dout),
                  ("dq", dq), ("dk", dk), ("dv", dv), ("drel", drel)):
        setattr(p, f"{nm}_stride_t", t.stride(0))
        setattr(p, f"{nm}_stride_h", t.stride(1))
    p.lse_stride_h, p.lse_stride_t = lse.stride(0), lse.stride(1)
    p.total_q, p.total_k = q.shape[0], k.shape[0]
    p.batch = cu_seqlens_q.numel() - 1
    p.n_heads, p.kv_heads, p.head_dim, p.rel_extent = n_heads, kv_heads, _ops.HEAD_DIM, rel_extent
    p.causal = 1 if causal else 0
    p.window_left = window_left
    p.causal_align = _ops.ALIGN[causal_align]
    p.max_seqlen_q = int(max_seqlen_q) if max_seqlen_q else 0
    p.max_seqlen_k = int(max_seqlen_k) if max_seqlen_k else 0
    p.dtype = _lib.IFA4_DTYPE_BF16
    p.softmax_scale = scale
    with torch.cuda.device(q.device):
        nbytes = ctypes.c_size_t(0)
        _lib.check(_lib.lib().ifa4_backward_workspace_size(ctypes.byref(p), ctypes.byref(nbytes)))
        if nbytes.value and (workspace is None or workspace.numel() * workspace.element_size() < nbytes.value):
            workspace = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
        ws_ptr = workspace.data_ptr() if nbytes.value else 0
        ws_len = workspace.numel() * workspace.element_size() if nbytes.value else 0
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.lib().ifa4_backward_launch(ctypes.byref(p), ctypes.c_void_p(ws_ptr),
                                                   ctypes.c_size_t(ws_len), ctypes.c_void_p(stream)))
    return dq, dk, dv, drel


class RelAttnFunction(torch.autograd.Function):
    """Prefill forward with saved LSE; backward through ``inkling_fa4_rel_attention_backward``."""

    @staticmethod
    def forward(ctx, q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                rel_extent, causal, window_size, softmax_scale, causal_align):
        out, lse = _ops.prefill(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                max_seqlen_k, rel_extent, causal=causal, window_size=window_size,
                                softmax_scale=softmax_scale, causal_align=causal_align,
                                return_lse=True)
        ctx.save_for_backward(q, k, v, rel_logits, out, lse, cu_seqlens_q, cu_seqlens_k)
        ctx.args = (max_seqlen_q, max_seqlen_k, rel_extent, causal, window_size, softmax_scale,
                    causal_align)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, rel, out, lse, cu_q, cu_k = ctx.saved_tensors
        max_q, max_k, rel_extent, causal, window_size, scale, align = ctx.args
        dq, dk, dv, drel = inkling_fa4_rel_attention_backward(
            dout.contiguous(), q, k, v, rel, out, lse, cu_q, cu_k, max_q, max_k, rel_extent,
            causal=causal, window_size=window_size, softmax_scale=scale, causal_align=align)
        return dq, dk, dv, drel, None, None, None, None, None, None, None, None, None


def inkling_fa4_rel_attention(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                              max_seqlen_k, rel_extent, causal=True, window_size=(-1, -1),
                              softmax_scale=None, causal_align="reference"):
    """Differentiable prefill: the forward of ``inkling_fa4_rel_attention_triton`` with
    gradients for q, k, v and rel_logits."""
    return RelAttnFunction.apply(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                 max_seqlen_k, rel_extent, causal, window_size, softmax_scale,
                                 causal_align)


__all__ = ["inkling_fa4_rel_attention_backward", "inkling_fa4_rel_attention", "RelAttnFunction"]
