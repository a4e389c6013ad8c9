"""Host side of the drop-in API: argument checks mirroring the reference call surface, stride
handling, and the calls through the C ABI (``_lib``).  Launches go on torch's current CUDA
stream of the input's device; nothing here synchronises with the device, so the calls can be
captured in a CUDA graph."""
from __future__ import annotations

import ctypes

import torch

from . import _lib

HEAD_DIM = 128
ALIGN = {"reference": _lib.IFA4_ALIGN_REFERENCE, "bottom_right": _lib.IFA4_ALIGN_BOTTOM_RIGHT}
# Launch through the torch operators (csrc/ifa4_torch_ops.cpp) when they are built; False (or an
# unbuilt operator library) keeps every launch on the ctypes calls of the same C ABI.
USE_TORCH_OPS = True


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """q/k/v go through TMA: last stride 1, other strides multiples of 8 elements (16 bytes),
    16-byte aligned base.  Anything else is copied to a contiguous tensor."""
    ok = (t.stride(-1) == 1 and all(s > 0 and s % 8 == 0 for s in t.stride()[:-1])
          and t.data_ptr() % 16 == 0)
    return t if ok else t.contiguous()


def _check_inputs(name, q, k, v, rel_logits, cu_q, cu_k, rel_extent, n_heads, kv_heads,
                  head_dim, window_size, causal_align, block_table=None):
    paged = block_table is not None
    tensors = [("q", q), ("k", k), ("v", v), ("rel_logits", rel_logits),
               ("cu_seqlens_q", cu_q), ("cu_seqlens_k", cu_k)]
    if paged:
        tensors.append(("block_table", block_table))
    for nm, t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name}: {nm} must be a torch.Tensor")
        if not t.is_cuda:
            raise ValueError(f"{name}: {nm} must be a CUDA tensor (no CPU path exists)")
        if t.device != q.device:
            raise ValueError(f"{name}: {nm} is on {t.device}, q on {q.device}")
    for nm, t in (("q", q), ("k", k), ("v", v), ("rel_logits", rel_logits)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name}: {nm} must be bfloat16, got {t.dtype}")
        want = 4 if paged and nm in ("k", "v") else 3
        if t.dim() != want:
            raise ValueError(f"{name}: {nm} must be {want}-D"
                             + (" [num_pages, page_size, kv_heads, head_dim]" if want == 4 else ""))
    for nm, t in (("cu_seqlens_q", cu_q), ("cu_seqlens_k", cu_k)):
        if t.dtype != torch.int32 or t.dim() != 1 or t.numel() < 1:
            raise ValueError(f"{name}: {nm} must be a non-empty 1-D int32 tensor")
    if cu_q.numel() != cu_k.numel():
        raise ValueError(f"{name}: cu_seqlens_q and cu_seqlens_k differ in length")
    hdim = 2 if paged else 1  # kv head dimension of k / v
    if n_heads is None:
        n_heads = q.shape[1]
    if kv_heads is None:
        kv_heads = k.shape[hdim]
    if n_heads != q.shape[1] or kv_heads != k.shape[hdim] or v.shape[hdim] != kv_heads:
        raise ValueError(f"{name}: head counts disagree with tensor shapes")
    if n_heads % kv_heads != 0:
        raise ValueError(f"{name}: n_heads {n_heads} not a multiple of kv_heads {kv_heads}")
    if head_dim != HEAD_DIM or q.shape[-1] != HEAD_DIM or k.shape[-1] != HEAD_DIM or v.shape[-1] != HEAD_DIM:
        raise ValueError(f"{name}: head_dim must be {HEAD_DIM}")
    if k.shape[:-1] != v.shape[:-1]:
        raise ValueError(f"{name}: k and v differ in shape")
    if paged:
        ps = k.shape[1]
        if ps < 16 or ps & (ps - 1):
            raise ValueError(f"{name}: page_size {ps} must be a power of two >= 16")
        if (block_table.dtype != torch.int32 or block_table.dim() != 2
                or block_table.shape[0] != cu_q.numel() - 1
                or (block_table.shape[1] > 1 and block_table.stride(1) != 1)):
            raise ValueError(f"{name}: block_table must be int32 [batch, max_pages] with unit "
                             "last stride")
    if rel_logits.shape[0] != q.shape[0] or rel_logits.shape[1] != n_heads:
        raise ValueError(f"{name}: rel_logits must be [total_q, n_heads, >=rel_extent]")
    rel_extent = int(rel_extent)
    if rel_extent <= 0 or rel_logits.shape[2] < rel_extent:
        raise ValueError(f"{name}: rel_extent {rel_extent} out of range for rel_logits {tuple(rel_logits.shape)}")
    if causal_align not in ALIGN:
        raise ValueError(f"{name}: causal_align must be one of {sorted(ALIGN)}")
    window_left = int(window_size[0]) if window_size is not None else -1
    return n_heads, kv_heads, rel_extent, window_left


def _lse_buffer(q, n_heads, return_lse, lse):
    """fp32 [n_heads, total_q] log-sum-exp output (flash-attention's varlen layout)."""
    if lse is None and not return_lse:
        return None
    if lse is None:
        lse = torch.empty((n_heads, q.shape[0]), dtype=torch.float32, device=q.device)
    if lse.dtype != torch.float32 or lse.shape != (n_heads, q.shape[0]) or lse.device != q.device:
        raise ValueError("lse must be a float32 [n_heads, total_q] tensor on q's device")
    return lse


def _fill_lse(p, lse):
    if lse is None:
        p.lse, p.lse_stride_h, p.lse_stride_t = None, 0, 0
    else:
        p.lse, p.lse_stride_h, p.lse_stride_t = lse.data_ptr(), lse.stride(0), lse.stride(1)


def _fill_common(p, q, k, v, rel, out, cu_q, cu_k, n_heads, kv_heads, rel_extent, causal,
                 window_left, causal_align, block_table=None):
    p.q, p.k, p.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.rel, p.out = rel.data_ptr(), out.data_ptr()
    p.cu_seqlens_q, p.cu_seqlens_k = cu_q.data_ptr(), cu_k.data_ptr()
    p.q_stride_t, p.q_stride_h = q.stride(0), q.stride(1)
    p.k_stride_t, p.k_stride_h = k.stride(-3), k.stride(-2)
    p.v_stride_t, p.v_stride_h = v.stride(-3), v.stride(-2)
    p.rel_stride_t, p.rel_stride_h = rel.stride(0), rel.stride(1)
    p.out_stride_t, p.out_stride_h = out.stride(0), out.stride(1)
    p.total_q = q.shape[0]
    if block_table is None:
        p.total_k = k.shape[0]
        p.block_table, p.block_table_stride = None, 0
        p.k_stride_page = p.v_stride_page = p.page_size = p.num_pages = 0
    else:
        p.total_k = k.shape[0] * k.shape[1]
        p.block_table, p.block_table_stride = block_table.data_ptr(), block_table.stride(0)
        p.k_stride_page, p.v_stride_page = k.stride(0), v.stride(0)
        p.page_size, p.num_pages = k.shape[1], k.shape[0]
    p.batch = cu_q.numel() - 1
    p.n_heads, p.kv_heads, p.head_dim = n_heads, kv_heads, HEAD_DIM
    p.rel_extent = rel_extent
    p.causal = 1 if causal else 0
    p.window_left = window_left
    p.causal_align = ALIGN[causal_align]
    p.dtype = _lib.IFA4_DTYPE_BF16


def _prepare(name, q, k, v, rel_logits, cu_q, cu_k, rel_extent, causal, window_size, n_heads,
             kv_heads, head_dim, softmax_scale, causal_align, out, block_table=None):
    n_heads, kv_heads, rel_extent, window_left = _check_inputs(
        name, q, k, v, rel_logits, cu_q, cu_k, rel_extent, n_heads, kv_heads, head_dim,
        window_size, causal_align, block_table)
    if block_table is not None:
        # a paged cache is never copied: it must already suit TMA
        for nm, t in (("k", k), ("v", v)):
            if _tma_ready(t) is not t:
                raise ValueError(f"{name}: paged {nm} cache needs unit last stride, strides "
                                 "that are positive multiples of 8 elements, 16-byte alignment")
        q = _tma_ready(q)
    else:
        q, k, v = _tma_ready(q), _tma_ready(k), _tma_ready(v)
    rel = rel_logits if rel_logits.stride(-1) == 1 else rel_logits.contiguous()
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    else:
        if out.shape != q.shape or out.dtype != q.dtype or out.device != q.device:
            raise ValueError(f"{name}: out must match q in shape, dtype and device")
        if out.stride(-1) != 1 or any(s % 8 for s in out.stride()[:-1]) or out.data_ptr() % 16:
            raise ValueError(f"{name}: out needs unit last stride, strides multiple of 8, 16-B alignment")
    scale = (1.0 / HEAD_DIM) if softmax_scale is None else float(softmax_scale)
    if not scale > 0:
        raise ValueError(f"{name}: softmax_scale must be > 0")
    return q, k, v, rel, out, n_heads, kv_heads, rel_extent, window_left, scale


def _table(block_table):
    """Unit last stride, and never a NULL pointer (NULL means "not paged" in the C ABI): an empty
    table becomes one column of -1 entries, which read as zero keys."""
    if block_table is None or not isinstance(block_table, torch.Tensor):
        return block_table
    if block_table.dim() == 2 and block_table.numel() == 0 and block_table.shape[0] > 0:
        return torch.full((block_table.shape[0], 1), -1, dtype=torch.int32,
                          device=block_table.device)
    return block_table if block_table.stride(-1) == 1 else block_table.contiguous()


@torch.no_grad()
def prefill(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
            rel_extent, causal=True, window_size=(-1, -1), n_heads=None, kv_heads=None,
            head_dim=HEAD_DIM, softmax_scale=None, causal_align="reference", out=None,
            tile_config=0, return_lse=False, lse=None, block_table=None, out_peers=None,
            kv_splits=0, workspace=None):
    """``out_peers``: optional device addresses (valid in this process) of the element that
    corresponds to ``out[0, 0, 0]`` in other GPUs' output buffers laid out like ``out``'s; the
    kernel stores every output row there too (see ``inkling_fa4.sharding.PeerOutputs``).
    ``kv_splits``: 0 lets the library split each query tile's KV range over several CTAs when
    the launch is too small to fill the GPU (the partials go to ``workspace``, allocated here if
    not given or too small); 1 never splits; > 1 forces that many splits."""
    block_table = _table(block_table)
    q, k, v, rel, out, n_heads, kv_heads, rel_extent, window_left, scale = _prepare(
        "prefill", q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, rel_extent, causal,
        window_size, n_heads, kv_heads, head_dim, softmax_scale, causal_align, out, block_table)
    lse = _lse_buffer(q, n_heads, return_lse, lse)
    ops = _lib.torch_ops() if USE_TORCH_OPS and not out_peers else None
    if ops is not None:  # one dispatcher call: parameter block, stream, workspace, launch
        rc = ops.prefill_(q, k, v, rel, out, cu_seqlens_q, cu_seqlens_k, lse, block_table,
                          workspace, rel_extent, bool(causal), window_left, ALIGN[causal_align],
                          int(max_seqlen_q) if max_seqlen_q else 0,
                          int(max_seqlen_k) if max_seqlen_k else 0, scale, int(tile_config),
                          int(kv_splits))
        if rc:
            _lib.check(rc)
        return (out, lse) if lse is not None else out
    p = _lib.PrefillParams()
    _fill_lse(p, lse)
    _fill_common(p, q, k, v, rel, out, cu_seqlens_q, cu_seqlens_k, n_heads, kv_heads,
                 rel_extent, causal, window_left, causal_align, block_table)
    p.max_seqlen_q = int(max_seqlen_q) if max_seqlen_q else 0
    p.softmax_scale = scale
    p.tile_config = int(tile_config)
    p.kv_splits = int(kv_splits)
    p.max_seqlen_k = int(max_seqlen_k) if max_seqlen_k else 0
    peers = None
    if out_peers:
        if len(out_peers) > _lib.MAX_OUT_PEERS:
            raise ValueError(f"prefill: at most {_lib.MAX_OUT_PEERS} out_peers")
        peers = (ctypes.c_void_p * len(out_peers))(*[int(x) for x in out_peers])
        p.out_peers = ctypes.cast(peers, ctypes.POINTER(ctypes.c_void_p))
        p.n_out_peers = len(out_peers)
    L = _lib.lib()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if p.kv_splits == 1 or p.n_out_peers > 0:
            _lib.check(L.ifa4_prefill_launch(ctypes.byref(p), ctypes.c_void_p(stream)))
        else:
            nbytes = ctypes.c_size_t(0)
            _lib.check(L.ifa4_prefill_workspace_size(ctypes.byref(p), ctypes.byref(nbytes)))
            need = int(nbytes.value)
            if need > 0 and (workspace is None
                             or workspace.numel() * workspace.element_size() < need):
                workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
            ws_ptr = workspace.data_ptr() if need > 0 else 0
            _lib.check(L.ifa4_prefill_launch_ws(ctypes.byref(p), ctypes.c_void_p(ws_ptr),
                                                ctypes.c_size_t(need), ctypes.c_void_p(stream)))
    return (out, lse) if lse is not None else out


def _decode_params(q, k, v, rel, out, cu_q, cu_k, n_heads, kv_heads, rel_extent, causal,
                   window_left, causal_align, max_seqlen_k, scale, num_splits, chunk_len,
                   block_table=None):
    p = _lib.DecodeParams()
    _fill_common(p, q, k, v, rel, out, cu_q, cu_k, n_heads, kv_heads, rel_extent, causal,
                 window_left, causal_align, block_table)
    p.max_seqlen_k = int(max_seqlen_k) if max_seqlen_k else 0
    p.softmax_scale = scale
    p.num_splits = int(num_splits)
    p.chunk_len = int(chunk_len)
    _fill_lse(p, None)
    return p


def decode_plan(p) -> tuple[int, int, int]:
    """(workspace bytes, num_splits, chunk_len) the library resolves for these parameters."""
    nbytes = ctypes.c_size_t(0)
    ns, cl = ctypes.c_int32(0), ctypes.c_int32(0)
    _lib.check(_lib.lib().ifa4_decode_workspace_size(ctypes.byref(p), ctypes.byref(nbytes),
                                                     ctypes.byref(ns), ctypes.byref(cl)))
    return int(nbytes.value), int(ns.value), int(cl.value)


@torch.no_grad()
def decode(q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
           rel_extent, causal=True, window_size=(-1, -1), n_heads=None, kv_heads=None,
           head_dim=HEAD_DIM, softmax_scale=None, causal_align="reference", out=None,
           num_splits=0, chunk_len=0, workspace=None, return_lse=False, lse=None,
           block_table=None):
    block_table = _table(block_table)
    q, k, v, rel, out, n_heads, kv_heads, rel_extent, window_left, scale = _prepare(
        "decode", q, k, v, rel_logits, cu_seqlens_q, cu_seqlens_k, rel_extent, causal,
        window_size, n_heads, kv_heads, head_dim, softmax_scale, causal_align, out, block_table)
    lse = _lse_buffer(q, n_heads, return_lse, lse)
    if q.shape[0] != cu_seqlens_q.numel() - 1:
        raise ValueError("decode: expects exactly one query token per sequence")
    if q.stride(0) % 2 or q.stride(1) % 2:
        q = q.contiguous()
    ops = _lib.torch_ops() if USE_TORCH_OPS else None
    if ops is not None:  # one dispatcher call: parameter block, stream, workspace, launch
        rc = ops.decode_(q, k, v, rel, out, cu_seqlens_q, cu_seqlens_k, lse, block_table,
                         workspace, rel_extent, bool(causal), window_left, ALIGN[causal_align],
                         int(max_seqlen_k) if max_seqlen_k else 0, scale, int(num_splits),
                         int(chunk_len))
        if rc:
            _lib.check(rc)
        return (out, lse) if lse is not None else out
    p = _decode_params(q, k, v, rel, out, cu_seqlens_q, cu_seqlens_k, n_heads, kv_heads,
                       rel_extent, causal, window_left, causal_align, max_seqlen_k, scale,
                       num_splits, chunk_len, block_table)
    _fill_lse(p, lse)
    with torch.cuda.device(q.device):
        nbytes, _, _ = decode_plan(p)
        if nbytes > 0 and (workspace is None or workspace.numel() * workspace.element_size() < nbytes):
            workspace = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        ws_ptr = workspace.data_ptr() if nbytes > 0 else 0
        ws_len = workspace.numel() * workspace.element_size() if nbytes > 0 else 0
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.lib().ifa4_decode_launch(ctypes.byref(p), ctypes.c_void_p(ws_ptr),
                                                 ctypes.c_size_t(ws_len), ctypes.c_void_p(stream)))
    return (out, lse) if lse is not None else out
