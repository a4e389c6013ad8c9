// torch operators over the C ABI: inkling_fa4::prefill_ and inkling_fa4::decode_.
//
// The Python package checks its arguments (the reference's call surface and error messages) and
// then calls one of these operators, which fills the IFA4 parameter block from the tensors'
// pointers and element strides, takes torch's current CUDA stream of the tensors' device, sizes
// and allocates the workspace through torch's caching allocator when the launch needs one, and
// calls ifa4_prefill_launch_ws / ifa4_decode_launch.  This replaces about forty ctypes field
// assignments and two foreign calls per attention call with one dispatcher call (the host cost
// that bounds small launches).  The operators return the C ABI's status code; the caller turns a
// nonzero code into an exception with ifa4_last_error_string().
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "../../include/inkling_fa4.h"

namespace {

void fill_common(IFA4PrefillParams* p, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                 const at::Tensor& rel, const at::Tensor& out, const at::Tensor& cu_q,
                 const at::Tensor& cu_k, const c10::optional<at::Tensor>& block_table,
                 int64_t rel_extent, bool causal, int64_t window_left, int64_t causal_align) {
  p->q = q.data_ptr();
  p->k = k.data_ptr();
  p->v = v.data_ptr();
  p->rel = rel.data_ptr();
  p->out = out.data_ptr();
  p->cu_seqlens_q = static_cast<const int32_t*>(cu_q.data_ptr());
  p->cu_seqlens_k = static_cast<const int32_t*>(cu_k.data_ptr());
  p->q_stride_t = q.stride(0);
  p->q_stride_h = q.stride(1);
  p->k_stride_t = k.stride(-3);
  p->k_stride_h = k.stride(-2);
  p->v_stride_t = v.stride(-3);
  p->v_stride_h = v.stride(-2);
  p->rel_stride_t = rel.stride(0);
  p->rel_stride_h = rel.stride(1);
  p->out_stride_t = out.stride(0);
  p->out_stride_h = out.stride(1);
  p->total_q = q.size(0);
  p->batch = static_cast<int32_t>(cu_q.numel() - 1);
  p->n_heads = static_cast<int32_t>(q.size(1));
  p->kv_heads = static_cast<int32_t>(k.size(-2));
  p->head_dim = 128;
  p->rel_extent = static_cast<int32_t>(rel_extent);
  p->causal = causal ? 1 : 0;
  p->window_left = static_cast<int32_t>(window_left);
  p->causal_align = static_cast<int32_t>(causal_align);
  p->dtype = IFA4_DTYPE_BF16;
  if (block_table.has_value()) {
    const at::Tensor& bt = *block_table;
    p->total_k = k.size(0) * k.size(1);
    p->block_table = static_cast<const int32_t*>(bt.data_ptr());
    p->block_table_stride = bt.stride(0);
    p->k_stride_page = k.stride(0);
    p->v_stride_page = v.stride(0);
    p->page_size = static_cast<int32_t>(k.size(1));
    p->num_pages = static_cast<int32_t>(k.size(0));
  } else {
    p->total_k = k.size(0);
  }
}

int64_t prefill_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                   const at::Tensor& rel, const at::Tensor& out, const at::Tensor& cu_q,
                   const at::Tensor& cu_k, const c10::optional<at::Tensor>& lse,
                   const c10::optional<at::Tensor>& block_table,
                   const c10::optional<at::Tensor>& workspace, int64_t rel_extent, bool causal,
                   int64_t window_left, int64_t causal_align, int64_t max_seqlen_q,
                   int64_t max_seqlen_k, double softmax_scale, int64_t tile_config,
                   int64_t kv_splits) {
  const c10::cuda::CUDAGuard guard(q.device());
  IFA4PrefillParams p{};
  fill_common(&p, q, k, v, rel, out, cu_q, cu_k, block_table, rel_extent, causal, window_left,
              causal_align);
  if (lse.has_value()) {
    p.lse = static_cast<float*>(lse->data_ptr());
    p.lse_stride_h = lse->stride(0);
    p.lse_stride_t = lse->stride(1);
  }
  p.max_seqlen_q = static_cast<int32_t>(max_seqlen_q);
  p.max_seqlen_k = static_cast<int32_t>(max_seqlen_k);
  p.softmax_scale = static_cast<float>(softmax_scale);
  p.tile_config = static_cast<int32_t>(tile_config);
  p.kv_splits = static_cast<int32_t>(kv_splits);
  void* stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  if (p.kv_splits == 1) return ifa4_prefill_launch(&p, stream);
  size_t need = 0;
  int rc = ifa4_prefill_workspace_size(&p, &need);
  if (rc) return rc;
  at::Tensor ws;
  if (need > 0) {
    if (workspace.has_value() && static_cast<size_t>(workspace->nbytes()) >= need)
      ws = *workspace;
    else
      ws = at::empty({static_cast<int64_t>(need)}, q.options().dtype(at::kByte));
  }
  return ifa4_prefill_launch_ws(&p, need > 0 ? ws.data_ptr() : nullptr, need, stream);
}

int64_t decode_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                  const at::Tensor& rel, const at::Tensor& out, const at::Tensor& cu_q,
                  const at::Tensor& cu_k, const c10::optional<at::Tensor>& lse,
                  const c10::optional<at::Tensor>& block_table,
                  const c10::optional<at::Tensor>& workspace, int64_t rel_extent, bool causal,
                  int64_t window_left, int64_t causal_align, int64_t max_seqlen_k,
                  double softmax_scale, int64_t num_splits, int64_t chunk_len) {
  const c10::cuda::CUDAGuard guard(q.device());
  // the decode parameter block starts with the same fields as the prefill one
  IFA4PrefillParams common{};
  fill_common(&common, q, k, v, rel, out, cu_q, cu_k, block_table, rel_extent, causal,
              window_left, causal_align);
  IFA4DecodeParams p{};
  p.q = common.q;
  p.k = common.k;
  p.v = common.v;
  p.rel = common.rel;
  p.out = common.out;
  p.cu_seqlens_q = common.cu_seqlens_q;
  p.cu_seqlens_k = common.cu_seqlens_k;
  p.q_stride_t = common.q_stride_t;
  p.q_stride_h = common.q_stride_h;
  p.k_stride_t = common.k_stride_t;
  p.k_stride_h = common.k_stride_h;
  p.v_stride_t = common.v_stride_t;
  p.v_stride_h = common.v_stride_h;
  p.rel_stride_t = common.rel_stride_t;
  p.rel_stride_h = common.rel_stride_h;
  p.out_stride_t = common.out_stride_t;
  p.out_stride_h = common.out_stride_h;
  p.total_q = common.total_q;
  p.total_k = common.total_k;
  p.batch = common.batch;
  p.n_heads = common.n_heads;
  p.kv_heads = common.kv_heads;
  p.head_dim = common.head_dim;
  p.rel_extent = common.rel_extent;
  p.causal = common.causal;
  p.window_left = common.window_left;
  p.causal_align = common.causal_align;
  p.dtype = common.dtype;
  p.block_table = common.block_table;
  p.block_table_stride = common.block_table_stride;
  p.k_stride_page = common.k_stride_page;
  p.v_stride_page = common.v_stride_page;
  p.page_size = common.page_size;
  p.num_pages = common.num_pages;
  if (lse.has_value()) {
    p.lse = static_cast<float*>(lse->data_ptr());
    p.lse_stride_h = lse->stride(0);
    p.lse_stride_t = lse->stride(1);
  }
  p.max_seqlen_k = static_cast<int32_t>(max_seqlen_k);
  p.softmax_scale = static_cast<float>(softmax_scale);
  p.num_splits = static_cast<int32_t>(num_splits);
  p.chunk_len = static_cast<int32_t>(chunk_len);
  void* stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  size_t need = 0;
  int rc = ifa4_decode_workspace_size(&p, &need, nullptr, nullptr);
  if (rc) return rc;
  at::Tensor ws;
  if (need > 0) {
    if (workspace.has_value() && static_cast<size_t>(workspace->nbytes()) >= need)
      ws = *workspace;
    else
      ws = at::empty({static_cast<int64_t>(need)}, q.options().dtype(at::kByte));
  }
  return ifa4_decode_launch(&p, need > 0 ? ws.data_ptr() : nullptr,
                            need > 0 ? static_cast<size_t>(ws.nbytes()) : 0, stream);
}

}  // namespace

TORCH_LIBRARY(inkling_fa4, m) {
  m.def("prefill_(Tensor q, Tensor k, Tensor v, Tensor rel, Tensor(a!) out, Tensor cu_q, "
        "Tensor cu_k, Tensor(b!)? lse, Tensor? block_table, Tensor? workspace, int rel_extent, "
        "bool causal, int window_left, int causal_align, int max_seqlen_q, int max_seqlen_k, "
        "float softmax_scale, int tile_config, int kv_splits) -> int");
  m.def("decode_(Tensor q, Tensor k, Tensor v, Tensor rel, Tensor(a!) out, Tensor cu_q, "
        "Tensor cu_k, Tensor(b!)? lse, Tensor? block_table, Tensor? workspace, int rel_extent, "
        "bool causal, int window_left, int causal_align, int max_seqlen_k, float softmax_scale, "
        "int num_splits, int chunk_len) -> int");
}

TORCH_LIBRARY_IMPL(inkling_fa4, CUDA, m) {
  m.impl("prefill_", &prefill_op);
  m.impl("decode_", &decode_op);
}
