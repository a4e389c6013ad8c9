// C ABI of the inkling_fa4 sm_100a kernels: argument validation, TMA descriptor encoding,
// launch planning, error reporting.  Declared in include/inkling_fa4.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "../../include/inkling_fa4.h"
#include "ifa4_internal.h"
#include "ifa4_ptx.cuh"

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(IFA4_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Device status word: kernels OR IFA4 status bits into it when they abandon a bounded wait.
__device__ int g_ifa4_device_status;

// Exercises the bounded-wait path of the kernels on a barrier that nothing ever arrives on:
// warp 0 (one thread) gives up after timeout_ns and raises kStatusSelfTestTimeout; warp 1
// (warp-collective wait) has ten times the limit and must leave through the abort flag that
// warp 0 raised, never through its own timeout (kStatusSelfTestOwnTimeout).
__global__ void __launch_bounds__(64) ifa4_selftest_wait_kernel(int* status,
                                                                unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    ifa4::mbar_init(&bar, 1);
    abort_flag = 0;
    ifa4::fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    if ((threadIdx.x & 31) == 0) {
      const ifa4::AbortCtx ab{&abort_flag, status, ifa4::kStatusSelfTestTimeout};
      ifa4::mbar_wait(&bar, 0, ab, timeout_ns);
    }
  } else {
    const ifa4::AbortCtx ab{&abort_flag, status, ifa4::kStatusSelfTestOwnTimeout};
    ifa4::mbar_wait_warp(&bar, 0, ab, 10 * timeout_ns);
  }
  __syncthreads();
  if (threadIdx.x == 0) ifa4::mbar_arrive(&bar);  // complete the phase before the CTA exits
}

// Read-only HBM stream (measurement hook): every thread keeps four 16-byte non-coherent loads
// in flight per iteration over a grid-strided range and folds them into one word, which is
// written out only if it equals an unlikely constant (so the loads cannot be dropped).
__global__ void __launch_bounds__(512) ifa4_read_stream_kernel(const uint4* __restrict__ src,
                                                               unsigned long long n16,
                                                               uint32_t* sink) {
  const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
  unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t acc = 0;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = ifa4::ldg_nc_v4(src + i), b = ifa4::ldg_nc_v4(src + i + stride);
    const uint4 c = ifa4::ldg_nc_v4(src + i + 2 * stride), d = ifa4::ldg_nc_v4(src + i + 3 * stride);
    acc ^= (a.x ^ a.y ^ a.z ^ a.w) ^ (b.x ^ b.y ^ b.z ^ b.w) ^ (c.x ^ c.y ^ c.z ^ c.w) ^
           (d.x ^ d.y ^ d.z ^ d.w);
  }
  for (; i < n16; i += stride) {
    const uint4 a = ifa4::ldg_nc_v4(src + i);
    acc ^= a.x ^ a.y ^ a.z ^ a.w;
  }
  if (acc == 0x9e3779b9u) atomicAdd(sink, 1u);
}

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {nullptr};
int g_sm_count[kMaxDevices] = {0};
std::mutex g_mu;

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(IFA4_ERR_UNSUPPORTED, "device ordinal %d", *dev);
  return IFA4_OK;
}

int device_status_ptr(int** out) {
  int dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ifa4_device_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  *out = g_status_ptr[dev];
  return IFA4_OK;
}

int sm_count(int* out) {
  int dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    g_sm_count[dev] = n;
  }
  *out = g_sm_count[dev];
  return IFA4_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* fn) {
  static EncodeTiledFn cached = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q != cudaDriverEntryPointSuccess) err = cudaErrorNotSupported;
    cached = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (err != cudaSuccess || cached == nullptr)
    return cuda_fail(err == cudaSuccess ? cudaErrorNotSupported : err,
                     "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
  *fn = cached;
  return IFA4_OK;
}

// [rows, heads, 128] bf16 with element strides (st, sh), boxes of 64 dims x 1 head x box_rows,
// 128-byte swizzle; out-of-range rows read as zero.
int encode_rows_heads_dims(CUtensorMap* map, const void* base, int64_t rows, int64_t heads,
                           int64_t st, int64_t sh, uint32_t box_rows, const char* name) {
  EncodeTiledFn fn;
  int rc = get_encode_fn(&fn);
  if (rc) return rc;
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(sh) * 2, static_cast<cuuint64_t>(st) * 2};
  cuuint32_t box[3] = {64, 1, box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(IFA4_ERR_UNSUPPORTED,
                "cuTensorMapEncodeTiled(%s) failed with CUresult %d (rows=%lld heads=%lld "
                "stride_t=%lld stride_h=%lld)",
                name, static_cast<int>(r), static_cast<long long>(rows),
                static_cast<long long>(heads), static_cast<long long>(st),
                static_cast<long long>(sh));
  return IFA4_OK;
}

// Paged cache [pages, page_size, heads, 128] bf16 with element strides (sp, st, sh): 4-D boxes
// of 64 dims x 1 head x box_rows x 1 page, 128-byte swizzle; out-of-range pages read as zero.
int encode_paged(CUtensorMap* map, const void* base, int64_t pages, int64_t page_size,
                 int64_t heads, int64_t sp, int64_t st, int64_t sh, uint32_t box_rows,
                 const char* name) {
  EncodeTiledFn fn;
  int rc = get_encode_fn(&fn);
  if (rc) return rc;
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(page_size),
                        static_cast<cuuint64_t>(pages)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(sh) * 2, static_cast<cuuint64_t>(st) * 2,
                           static_cast<cuuint64_t>(sp) * 2};
  cuuint32_t box[4] = {64, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(IFA4_ERR_UNSUPPORTED,
                "cuTensorMapEncodeTiled(%s, paged) failed with CUresult %d (pages=%lld "
                "page_size=%lld heads=%lld stride_page=%lld stride_t=%lld stride_h=%lld)",
                name, static_cast<int>(r), static_cast<long long>(pages),
                static_cast<long long>(page_size), static_cast<long long>(heads),
                static_cast<long long>(sp), static_cast<long long>(st), static_cast<long long>(sh));
  return IFA4_OK;
}

int log2_exact(int64_t x) {
  int s = 0;
  while ((int64_t{1} << s) < x) ++s;
  return s;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Checks shared by prefill and decode.
template <class P>
int validate_common(const P* p, const char* what) {
  if (p == nullptr) return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: params is NULL", what);
  if (p->dtype != IFA4_DTYPE_BF16)
    return fail(IFA4_ERR_UNSUPPORTED, "%s: dtype %d unsupported (bf16 only)", what, p->dtype);
  if (p->head_dim != ifa4::kHeadDim)
    return fail(IFA4_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (128 only)", what, p->head_dim);
  if (p->batch < 0 || p->total_q < 0 || p->total_k < 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: negative batch/total", what);
  if (p->n_heads <= 0 || p->kv_heads <= 0 || p->n_heads % p->kv_heads != 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: n_heads %d must be a positive multiple of kv_heads %d",
                what, p->n_heads, p->kv_heads);
  if (p->rel_extent <= 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: rel_extent must be > 0", what);
  if (!(p->softmax_scale > 0.f))
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: softmax_scale must be > 0", what);
  if (p->causal_align != IFA4_ALIGN_REFERENCE && p->causal_align != IFA4_ALIGN_BOTTOM_RIGHT)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: causal_align %d", what, p->causal_align);
  if (p->batch == 0 || p->total_q == 0) return IFA4_OK;
  if (!p->q || !p->k || !p->v || !p->rel || !p->out || !p->cu_seqlens_q || !p->cu_seqlens_k)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: null tensor pointer", what);
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out))
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: q/k/v/out must be 16-byte aligned", what);
  const int64_t s8[] = {p->q_stride_t, p->q_stride_h, p->k_stride_t, p->k_stride_h,
                        p->v_stride_t, p->v_stride_h, p->out_stride_t, p->out_stride_h};
  for (int64_t s : s8)
    if (s <= 0 || (s % 8) != 0)
      return fail(IFA4_ERR_INVALID_ARGUMENT,
                  "%s: q/k/v/out token and head strides must be positive multiples of 8 elements",
                  what);
  if (p->rel_stride_t < 0 || p->rel_stride_h < 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: negative rel strides", what);
  if (p->batch > 65535) return fail(IFA4_ERR_UNSUPPORTED, "%s: batch > 65535", what);
  if (p->n_heads > 65535) return fail(IFA4_ERR_UNSUPPORTED, "%s: n_heads > 65535", what);
  if (p->block_table != nullptr) {
    if (p->page_size < 16 || p->page_size > (1 << 20) || (p->page_size & (p->page_size - 1)) != 0)
      return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: page_size %d must be a power of two in [16, 2^20]",
                  what, p->page_size);
    if (p->num_pages <= 0)
      return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: num_pages must be > 0", what);
    if (p->block_table_stride < 0)
      return fail(IFA4_ERR_INVALID_ARGUMENT, "%s: negative block_table_stride", what);
    if (p->k_stride_page <= 0 || p->k_stride_page % 8 != 0 || p->v_stride_page <= 0 ||
        p->v_stride_page % 8 != 0)
      return fail(IFA4_ERR_INVALID_ARGUMENT,
                  "%s: k/v page strides must be positive multiples of 8 elements", what);
  }
  return IFA4_OK;
}

// Tensor maps for K and V: [total_k, kv_heads, 128] with boxes of `tile_rows` rows, or the
// paged caches with boxes of min(page_size, tile_rows) rows.
template <class P>
int encode_kv(const P* p, uint32_t tile_rows, CUtensorMap* tk, CUtensorMap* tv) {
  int rc;
  if (p->block_table != nullptr) {
    const uint32_t box = p->page_size < static_cast<int>(tile_rows) ? p->page_size : tile_rows;
    if ((rc = encode_paged(tk, p->k, p->num_pages, p->page_size, p->kv_heads, p->k_stride_page,
                           p->k_stride_t, p->k_stride_h, box, "k")))
      return rc;
    return encode_paged(tv, p->v, p->num_pages, p->page_size, p->kv_heads, p->v_stride_page,
                        p->v_stride_t, p->v_stride_h, box, "v");
  }
  const int64_t krows = p->total_k > 0 ? p->total_k : 1;
  if ((rc = encode_rows_heads_dims(tk, p->k, krows, p->kv_heads, p->k_stride_t, p->k_stride_h,
                                   tile_rows, "k")))
    return rc;
  return encode_rows_heads_dims(tv, p->v, krows, p->kv_heads, p->v_stride_t, p->v_stride_h,
                                tile_rows, "v");
}

// Kernel-side paged fields (no-ops without a block table).
template <class P, class A>
void fill_paged(const P* p, uint32_t tile_rows, A* a) {
  a->block_table = p->block_table;
  if (p->block_table == nullptr) return;
  a->bt_stride = p->block_table_stride;
  a->page_shift = log2_exact(p->page_size);
  a->box_shift = log2_exact(p->page_size < static_cast<int>(tile_rows) ? p->page_size : tile_rows);
  a->num_pages = p->num_pages;
}

}  // namespace

extern "C" {

const char* ifa4_last_error_string(void) { return g_last_error; }

int32_t ifa4_abi_version(void) { return IFA4_ABI_VERSION; }

const char* ifa4_prefill_tile_config_name(int32_t tile_config) {
  static const char* names[ifa4::kPrefillNumTileConfigs] = {
      "sm100_q2x128_kv128_d128_ws12_default", "sm100_q2x128_kv128_d128_ws12_emu0of16",
      "sm100_q2x128_kv128_d128_ws12_emu2of16", "sm100_q2x128_kv128_d128_ws12_emu4of16",
      "sm100_q2x128_kv128_d128_ws12_emu6of16", "sm100_q2x128_kv128_d128_ws12_emu8of16",
      "sm100_q2x128_kv128_d128_ws12_h2x16of16", "sm100_q2x128_kv128_d128_ws12_h2x8of16",
      "sm100_q2x128_kv128_d128_ws12_emu4h2x8of16"};
  if (tile_config < 0 || tile_config >= ifa4::kPrefillNumTileConfigs) return "";
  return names[tile_config];
}

}  // extern "C"

namespace {
int prefill_launch_impl(const IFA4PrefillParams* p, void* workspace, size_t workspace_bytes,
                        bool ws_entry, size_t* ws_bytes_out, void* stream) {
  int rc = validate_common(p, "prefill");
  if (rc) return rc;
  if (ifa4::prefill_emulated_exp_columns(p->tile_config) < 0)
    return fail(IFA4_ERR_UNSUPPORTED, "prefill: tile_config %d unknown", p->tile_config);
  if (p->block_table != nullptr && !ifa4::prefill_paged_tile_config_ok(p->tile_config))
    return fail(IFA4_ERR_UNSUPPORTED, "prefill: tile_config %d has no paged-cache variant (0 to 3)",
                p->tile_config);
  if (p->kv_splits < 0 || p->kv_splits > IFA4_MAX_KV_SPLITS)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "prefill: kv_splits %d outside [0, %d]", p->kv_splits,
                IFA4_MAX_KV_SPLITS);
  if (!ws_entry && p->kv_splits > 1)
    return fail(IFA4_ERR_INVALID_ARGUMENT,
                "prefill: kv_splits > 1 needs a workspace (ifa4_prefill_launch_ws)");
  if (p->kv_splits > 1 && (p->tile_config != 0 || p->n_out_peers > 0))
    return fail(IFA4_ERR_UNSUPPORTED, "prefill: kv_splits > 1 needs tile_config 0 and no out_peers");
  if (ws_bytes_out) *ws_bytes_out = 0;
  if (p->batch == 0 || p->total_q == 0) return IFA4_OK;
  int* status = nullptr;
  if (!ws_bytes_out && (rc = device_status_ptr(&status))) return rc;

  ifa4::PrefillKernelArgs a{};
  a.rel = static_cast<const uint16_t*>(p->rel);
  a.out = static_cast<uint16_t*>(p->out);
  a.cu_q = p->cu_seqlens_q;
  a.cu_k = p->cu_seqlens_k;
  a.rel_st = p->rel_stride_t;
  a.rel_sh = p->rel_stride_h;
  a.out_st = p->out_stride_t;
  a.out_sh = p->out_stride_h;
  a.batch = p->batch;
  a.n_heads = p->n_heads;
  a.kv_heads = p->kv_heads;
  a.rel_extent = p->rel_extent;
  a.causal = p->causal ? 1 : 0;
  a.window_left = p->window_left < 0 ? -1 : p->window_left;
  a.align_bottom_right = p->causal_align == IFA4_ALIGN_BOTTOM_RIGHT;
  const int group = p->n_heads / p->kv_heads;
  a.pair_heads = (group % 2 == 0) ? 1 : 0;
  a.scale_log2 = p->softmax_scale * 1.4426950408889634f;
  a.bias_vec = aligned16(p->rel) && p->rel_stride_t % 8 == 0 && p->rel_stride_h % 8 == 0 &&
               p->rel_extent % 8 == 0;
  a.lse = p->lse;
  a.lse_sh = p->lse_stride_h;
  a.lse_st = p->lse_stride_t;
  fill_paged(p, 128, &a);
  a.v = static_cast<const uint16_t*>(p->v);
  a.v_st = p->v_stride_t;
  a.v_sh = p->v_stride_h;
  a.v_sp = p->v_stride_page;
  a.status = status;
  if (p->n_out_peers < 0 || p->n_out_peers > IFA4_MAX_OUT_PEERS)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "prefill: n_out_peers %d outside [0, %d]",
                p->n_out_peers, IFA4_MAX_OUT_PEERS);
  if (p->n_out_peers > 0 && p->out_peers == nullptr)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "prefill: out_peers is NULL");
  if (p->n_out_peers > 0 && (p->block_table != nullptr || p->tile_config != 0))
    return fail(IFA4_ERR_UNSUPPORTED, "prefill: out_peers needs contiguous K/V and tile_config 0");
  a.n_out_peers = p->n_out_peers;
  for (int i = 0; i < p->n_out_peers; ++i) {
    const void* pp = p->out_peers[i];
    if (pp == nullptr || !aligned16(pp))
      return fail(IFA4_ERR_INVALID_ARGUMENT, "prefill: out_peers[%d] must be a 16-byte aligned "
                  "device address", i);
    // byte distance in elements (both addresses are 16-byte aligned)
    a.out_peer_delta[i] = (reinterpret_cast<intptr_t>(pp) - reinterpret_cast<intptr_t>(p->out)) /
                          static_cast<intptr_t>(sizeof(uint16_t));
  }

  // Grid order: query slots fastest when one query tile's key range over all KV heads (K and V,
  // 512 bytes per key and head; the average sequence's keys, capped by the window) is more than
  // a third of the 126 MB L2 (measured at 32k: causal +1 %, chunked 8 x 18k +8 %; window 4096
  // and ragged <= 4k sequences, whose ranges fit, lose 2 % with it).
  {
    const int64_t keys = p->block_table != nullptr
                             ? static_cast<int64_t>(p->num_pages) * p->page_size
                             : p->total_k;
    int64_t span = (keys + p->batch - 1) / p->batch;
    if (p->window_left >= 0 && p->window_left + 256 < span) span = p->window_left + 256;
    a.q_fastest = span * p->kv_heads * 512 > (48LL << 20);
  }
  const int rows_per_cta = a.pair_heads ? 128 : 256;
  int64_t max_sq = p->max_seqlen_q > 0 ? p->max_seqlen_q : p->total_q;
  if (max_sq > p->total_q) max_sq = p->total_q;
  int64_t slots = (max_sq + rows_per_cta - 1) / rows_per_cta;
  // Query slots per (head slot, sequence): enough for the average sequence (longer ones
  // stride over their tiles, query slot i taking tiles i, i + slots, ... heaviest first, which pairs
  // heavy with light tiles), but at least four waves of CTAs.  With one sequence (or equal
  // lengths) this is the longest sequence's tile count: one tile set per CTA.
  {
    const int64_t avg_sq = (p->total_q + p->batch - 1) / p->batch;
    const int64_t avg_slots = (avg_sq + rows_per_cta - 1) / rows_per_cta;
    int sms = 148;
    if ((rc = sm_count(&sms))) return rc;
    const int64_t head_slots = a.pair_heads ? p->n_heads / 2 : p->n_heads;
    const int64_t per_z = head_slots * p->batch;
    const int64_t min_slots = (4LL * sms + per_z - 1) / per_z;
    int64_t want = avg_slots > min_slots ? avg_slots : min_slots;
    if (want < slots) slots = want;
  }
  if (slots < 1) slots = 1;
  if (slots > 65535) slots = 65535;
  // KV split (workspace entry point only): when the grid leaves SMs idle, each query tile's KV
  // tiles are shared among kv_splits CTAs and a merge kernel combines their partials.  Measured
  // on B200 (one sequence, Hq = Hkv = 4 at 2k / 4k / 8k tokens and GQA 8/2 at 4k; 1..16 splits):
  // a grid of more than half the SMs gains only from 2 splits (8k: 182 -> 167 us; GQA 8/2 at 4k:
  // 78 -> 77 us, 91 us with 3), a smaller one is best near two waves of CTAs (4k: 113 -> 85 us
  // with 5; 2k: 84 -> 50 us with 8), with at least 2 KV tiles per share of the heaviest query
  // tile, which sees at most the longest sequence's keys (the max_seqlen_k hint, else all keys;
  // the window bounds it).
  int kv_splits = p->kv_splits > 1 ? p->kv_splits : 1;
  if (ws_entry && p->kv_splits == 0 && p->tile_config == 0 && p->n_out_peers == 0) {
    int sms = 148;
    if ((rc = sm_count(&sms))) return rc;
    const int64_t head_slots = a.pair_heads ? p->n_heads / 2 : p->n_heads;
    const int64_t ctas = head_slots * p->batch * slots;
    int64_t span = p->max_seqlen_k > 0 ? p->max_seqlen_k
                   : p->block_table != nullptr ? static_cast<int64_t>(p->num_pages) * p->page_size
                                               : p->total_k;
    if (p->window_left >= 0 && p->window_left + 256 < span) span = p->window_left + 256;
    const int64_t kv_tiles = (span + 127) / 128;
    if (ctas < sms) {
      int64_t want = 2 * ctas > sms ? 2 : (2 * sms + ctas - 1) / ctas;
      if (want > kv_tiles / 2) want = kv_tiles / 2;
      if (want > IFA4_MAX_KV_SPLITS) want = IFA4_MAX_KV_SPLITS;
      if (want >= 2) kv_splits = static_cast<int>(want);
    }
  }
  if (static_cast<int64_t>(slots) * kv_splits > 65535)
    return fail(IFA4_ERR_UNSUPPORTED, "prefill: %lld query slots x %d KV splits exceed the grid",
                static_cast<long long>(slots), kv_splits);
  const size_t ws_need = kv_splits > 1 ? static_cast<size_t>(kv_splits) * p->total_q *
                                             p->n_heads * (128 + 1) * sizeof(float)
                                       : 0;
  if (ws_bytes_out) {  // planning only
    *ws_bytes_out = ws_need;
    return IFA4_OK;
  }
  if (ws_need > 0) {
    if (workspace == nullptr || workspace_bytes < ws_need)
      return fail(IFA4_ERR_WORKSPACE, "prefill: workspace of %zu bytes required, got %zu", ws_need,
                  workspace_bytes);
    if (!aligned16(workspace)) return fail(IFA4_ERR_WORKSPACE, "prefill: workspace must be 16-byte aligned");
  }
  a.kv_splits = kv_splits;
  a.total_q = p->total_q;
  if (kv_splits > 1) {
    a.ws_o = static_cast<float*>(workspace);
    a.ws_lse = a.ws_o + static_cast<size_t>(kv_splits) * p->total_q * p->n_heads * 128;
  }
  CUtensorMap tq, tk, tv;
  if ((rc = encode_rows_heads_dims(&tq, p->q, p->total_q, p->n_heads, p->q_stride_t,
                                   p->q_stride_h, 128, "q")))
    return rc;
  if ((rc = encode_kv(p, 128, &tk, &tv))) return rc;
  cudaError_t e = ifa4::launch_prefill_sm100(a, tq, tk, tv, static_cast<int>(slots),
                                             p->tile_config, static_cast<int>(max_sq),
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  if (kv_splits > 1) {
    e = ifa4::launch_prefill_combine_sm100(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "prefill combine launch");
  }
  return IFA4_OK;
}
}  // namespace

extern "C" {

int ifa4_prefill_launch(const IFA4PrefillParams* p, void* stream) {
  g_last_error[0] = '\0';
  return prefill_launch_impl(p, nullptr, 0, false, nullptr, stream);
}

int ifa4_prefill_workspace_size(const IFA4PrefillParams* p, size_t* bytes_out) {
  g_last_error[0] = '\0';
  if (bytes_out == nullptr) return fail(IFA4_ERR_INVALID_ARGUMENT, "prefill: bytes_out is NULL");
  return prefill_launch_impl(p, nullptr, 0, true, bytes_out, nullptr);
}

int ifa4_prefill_launch_ws(const IFA4PrefillParams* p, void* workspace, size_t workspace_bytes,
                           void* stream) {
  g_last_error[0] = '\0';
  return prefill_launch_impl(p, workspace, workspace_bytes, true, nullptr, stream);
}



static int decode_plan(const IFA4DecodeParams* p, int* num_splits, int* chunk_len,
                       size_t* ws_bytes) {
  const int group = p->n_heads / p->kv_heads;
  const int hpc = group < 16 ? group : 16;
  const int head_blocks = (group + hpc - 1) / hpc;
  const int64_t key_cap = p->block_table != nullptr
                              ? static_cast<int64_t>(p->num_pages) * p->page_size
                              : p->total_k;
  int64_t max_sk = p->max_seqlen_k > 0 ? p->max_seqlen_k : key_cap;
  if (max_sk > key_cap) max_sk = key_cap;
  if (max_sk < 1) max_sk = 1;
  int chunk = p->chunk_len;
  int splits = p->num_splits;
  if (chunk < 0 || (chunk % 64) != 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "decode: chunk_len must be a multiple of 64");
  if (splits < 0) return fail(IFA4_ERR_INVALID_ARGUMENT, "decode: num_splits < 0");
  if (chunk == 0) {
    // 2048-key chunks balance ragged lengths across CTAs; only when they would leave SMs idle
    // (small batches) are they shortened, to at most one CTA per SM (measured on B200 at batch 1
    // and 32k keys: 18 x 1856-key chunks (144 CTAs) 36 us, 19 x 1728 (152: four SMs run two)
    // 40 us, 64 x 256 (two CTA waves, each paying the pipeline start) 46 us).
    int sms = 148;
    int rc = sm_count(&sms);
    if (rc) return rc;
    const int64_t ctas_per_split = static_cast<int64_t>(p->batch) * p->kv_heads * head_blocks;
    chunk = 2048;
    if (ctas_per_split * ((max_sk + chunk - 1) / chunk) < sms) {
      const int64_t want_splits = sms / ctas_per_split > 0 ? sms / ctas_per_split : 1;
      int64_t c = (max_sk + want_splits - 1) / want_splits;
      c = (c + 63) / 64 * 64;
      chunk = static_cast<int>(c < 64 ? 64 : (c > 2048 ? 2048 : c));
    }
  }
  if (splits == 0) {
    int64_t s = (max_sk + chunk - 1) / chunk;
    if (s > 64) s = 64;
    splits = static_cast<int>(s < 1 ? 1 : s);
  }
  if (splits > 65535) return fail(IFA4_ERR_INVALID_ARGUMENT, "decode: num_splits > 65535");
  *num_splits = splits;
  *chunk_len = chunk;
  if (splits == 1) {
    *ws_bytes = 0;
  } else {
    const size_t parts = static_cast<size_t>(p->batch) * p->n_heads * splits;
    *ws_bytes = parts * 128 * sizeof(float) + parts * sizeof(float);
  }
  return IFA4_OK;
}

int ifa4_decode_workspace_size(const IFA4DecodeParams* p, size_t* bytes_out,
                               int32_t* num_splits_out, int32_t* chunk_len_out) {
  g_last_error[0] = '\0';
  int rc = validate_common(p, "decode");
  if (rc) return rc;
  if (bytes_out == nullptr) return fail(IFA4_ERR_INVALID_ARGUMENT, "decode: bytes_out is NULL");
  int splits = 1, chunk = 64;
  size_t ws = 0;
  if (p->batch > 0 && p->total_q > 0) {
    if ((rc = decode_plan(p, &splits, &chunk, &ws))) return rc;
  }
  *bytes_out = ws;
  if (num_splits_out) *num_splits_out = splits;
  if (chunk_len_out) *chunk_len_out = chunk;
  return IFA4_OK;
}

int ifa4_decode_launch(const IFA4DecodeParams* p, void* workspace, size_t workspace_bytes,
                       void* stream) {
  g_last_error[0] = '\0';
  int rc = validate_common(p, "decode");
  if (rc) return rc;
  if (p->batch == 0 || p->total_q == 0) return IFA4_OK;
  if (p->total_q != p->batch)
    return fail(IFA4_ERR_INVALID_ARGUMENT,
                "decode: expects exactly one query per sequence (total_q %lld != batch %d)",
                static_cast<long long>(p->total_q), p->batch);
  int splits, chunk;
  size_t ws = 0;
  if ((rc = decode_plan(p, &splits, &chunk, &ws))) return rc;
  if (ws > 0 && (workspace == nullptr || workspace_bytes < ws))
    return fail(IFA4_ERR_WORKSPACE, "decode: workspace of %zu bytes required, got %zu", ws,
                workspace_bytes);
  if (ws > 0 && (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return fail(IFA4_ERR_WORKSPACE, "decode: workspace must be 16-byte aligned");
  int* status = nullptr;
  if ((rc = device_status_ptr(&status))) return rc;

  ifa4::DecodeKernelArgs a{};
  a.q = static_cast<const uint16_t*>(p->q);
  a.rel = static_cast<const uint16_t*>(p->rel);
  a.out = static_cast<uint16_t*>(p->out);
  a.cu_q = p->cu_seqlens_q;
  a.cu_k = p->cu_seqlens_k;
  a.q_st = p->q_stride_t;
  a.q_sh = p->q_stride_h;
  a.rel_st = p->rel_stride_t;
  a.rel_sh = p->rel_stride_h;
  a.out_st = p->out_stride_t;
  a.out_sh = p->out_stride_h;
  a.batch = p->batch;
  a.n_heads = p->n_heads;
  a.kv_heads = p->kv_heads;
  a.rel_extent = p->rel_extent;
  a.causal = p->causal ? 1 : 0;
  a.window_left = p->window_left < 0 ? -1 : p->window_left;
  a.align_bottom_right = p->causal_align == IFA4_ALIGN_BOTTOM_RIGHT;
  a.group = p->n_heads / p->kv_heads;
  a.heads_per_cta = a.group < 16 ? a.group : 16;
  a.num_splits = splits;
  a.chunk_len = chunk;
  a.scale_log2 = p->softmax_scale * 1.4426950408889634f;
  if (ws > 0) {
    const size_t parts = static_cast<size_t>(p->batch) * p->n_heads * splits;
    a.ws_o = static_cast<float*>(workspace);
    a.ws_lse = a.ws_o + parts * 128;
  }
  a.lse = p->lse;
  a.lse_sh = p->lse_stride_h;
  a.lse_st = p->lse_stride_t;
  fill_paged(p, 64, &a);
  a.status = status;
  CUtensorMap tk, tv;
  if ((rc = encode_kv(p, 64, &tk, &tv))) return rc;
  cudaError_t e = ifa4::launch_decode_sm100(a, tk, tv, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return IFA4_OK;
}

// ---------------------------------------------------------------------------------------
// Decode without allocation: for callers that may not call cudaMalloc (an engine that
// reserved all device memory up front, or an FFI plugin with no access to its host's
// allocator).  The split-KV partials live in this file-scope array instead of a caller
// workspace; every GPU that loads the library holds it until the process exits.  In host code
// the symbol is only a stand-in, so the device address is looked up once per device
// (cudaGetSymbolAddress with that device current) and passed to the kernels.
// ---------------------------------------------------------------------------------------
}  // extern "C"

static __device__ __align__(256) float g_ifa4_decode_scratch[IFA4_NOALLOC_DECODE_SCRATCH_BYTES /
                                                              sizeof(float)];

namespace {
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// First call on a device: resolves the scratch array's device address for the current device.
int decode_scratch_ptr(void** out) {
  int dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ifa4_decode_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return IFA4_OK;
}
}  // namespace

extern "C" {

int ifa4_decode_launch_noalloc(const IFA4DecodeParams* p, void* stream) {
  g_last_error[0] = '\0';
  int rc = validate_common(p, "decode_noalloc");
  if (rc) return rc;
  if (p->batch == 0 || p->total_q == 0) return IFA4_OK;
  int splits, chunk;
  size_t ws = 0;
  if ((rc = decode_plan(p, &splits, &chunk, &ws))) return rc;
  const size_t per_split = static_cast<size_t>(p->batch) * p->n_heads * (128 + 1) * sizeof(float);
  if (ws > IFA4_NOALLOC_DECODE_SCRATCH_BYTES) {
    if (p->num_splits != 0)
      return fail(IFA4_ERR_WORKSPACE,
                  "decode_noalloc: num_splits %d needs %zu bytes of scratch; the static scratch "
                  "holds %u bytes (at most %zu splits for batch %d x %d heads)",
                  p->num_splits, ws, IFA4_NOALLOC_DECODE_SCRATCH_BYTES,
                  static_cast<size_t>(IFA4_NOALLOC_DECODE_SCRATCH_BYTES) / per_split, p->batch,
                  p->n_heads);
    // automatic plan: cap the split count so the partials fit (CTAs stride over the chunks)
    size_t fit = static_cast<size_t>(IFA4_NOALLOC_DECODE_SCRATCH_BYTES) / per_split;
    splits = fit >= 2 ? static_cast<int>(fit) : 1;
  }
  IFA4DecodeParams q = *p;
  q.num_splits = splits;
  q.chunk_len = chunk;
  void* scratch = nullptr;
  if (splits > 1 && (rc = decode_scratch_ptr(&scratch))) return rc;
  return ifa4_decode_launch(&q, scratch, splits > 1 ? IFA4_NOALLOC_DECODE_SCRATCH_BYTES : 0,
                            stream);
}

// ---------------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------------
}  // extern "C"

namespace {
int validate_backward(const IFA4BackwardParams* p) {
  if (p == nullptr) return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: params is NULL");
  if (p->dtype != IFA4_DTYPE_BF16)
    return fail(IFA4_ERR_UNSUPPORTED, "backward: dtype %d unsupported (bf16 only)", p->dtype);
  if (p->head_dim != ifa4::kHeadDim)
    return fail(IFA4_ERR_UNSUPPORTED, "backward: head_dim %d unsupported (128 only)", p->head_dim);
  if (p->batch < 0 || p->total_q < 0 || p->total_k < 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: negative batch/total");
  if (p->n_heads <= 0 || p->kv_heads <= 0 || p->n_heads % p->kv_heads != 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT,
                "backward: n_heads %d must be a positive multiple of kv_heads %d", p->n_heads,
                p->kv_heads);
  if (p->rel_extent <= 0) return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: rel_extent must be > 0");
  if (!(p->softmax_scale > 0.f))
    return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: softmax_scale must be > 0");
  if (p->causal_align != IFA4_ALIGN_REFERENCE && p->causal_align != IFA4_ALIGN_BOTTOM_RIGHT)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: causal_align %d", p->causal_align);
  if (p->batch == 0 || p->total_q == 0) return IFA4_OK;
  if (!p->q || !p->k || !p->v || !p->rel || !p->out || !p->dout || !p->lse || !p->dq ||
      !p->dk || !p->dv || !p->drel || !p->cu_seqlens_q || !p->cu_seqlens_k)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: null tensor pointer");
  const void* a16[] = {p->q, p->k, p->v, p->out, p->dout, p->dq, p->dk, p->dv};
  for (const void* ptr : a16)
    if (!aligned16(ptr))
      return fail(IFA4_ERR_INVALID_ARGUMENT,
                  "backward: q/k/v/out/dout/dq/dk/dv must be 16-byte aligned");
  const int64_t s8[] = {p->q_stride_t,    p->q_stride_h,  p->k_stride_t,  p->k_stride_h,
                        p->v_stride_t,    p->v_stride_h,  p->out_stride_t, p->out_stride_h,
                        p->dout_stride_t, p->dout_stride_h, p->dq_stride_t, p->dq_stride_h,
                        p->dk_stride_t,   p->dk_stride_h, p->dv_stride_t,  p->dv_stride_h};
  for (int64_t s : s8)
    if (s <= 0 || (s % 8) != 0)
      return fail(IFA4_ERR_INVALID_ARGUMENT,
                  "backward: q/k/v/out/dout/dq/dk/dv token and head strides must be positive "
                  "multiples of 8 elements");
  if (p->rel_stride_t < 0 || p->rel_stride_h < 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: negative rel strides");
  if (p->drel_stride_t <= 0 || p->drel_stride_h <= 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: drel strides must be positive");
  if (p->batch > 65535) return fail(IFA4_ERR_UNSUPPORTED, "backward: batch > 65535");
  if (p->n_heads > 65535) return fail(IFA4_ERR_UNSUPPORTED, "backward: n_heads > 65535");
  return IFA4_OK;
}

size_t backward_workspace_bytes(const IFA4BackwardParams* p) {
  return static_cast<size_t>(p->n_heads) * static_cast<size_t>(p->total_q) * sizeof(float);
}
}  // namespace

extern "C" {

int ifa4_backward_workspace_size(const IFA4BackwardParams* p, size_t* bytes_out) {
  g_last_error[0] = '\0';
  int rc = validate_backward(p);
  if (rc) return rc;
  if (bytes_out == nullptr) return fail(IFA4_ERR_INVALID_ARGUMENT, "backward: bytes_out is NULL");
  *bytes_out = (p->batch == 0 || p->total_q == 0) ? 0 : backward_workspace_bytes(p);
  return IFA4_OK;
}

int ifa4_backward_launch(const IFA4BackwardParams* p, void* workspace, size_t workspace_bytes,
                         void* stream) {
  g_last_error[0] = '\0';
  int rc = validate_backward(p);
  if (rc) return rc;
  if (p->batch == 0 || p->total_q == 0) return IFA4_OK;
  const size_t ws = backward_workspace_bytes(p);
  if (workspace == nullptr || workspace_bytes < ws)
    return fail(IFA4_ERR_WORKSPACE, "backward: workspace of %zu bytes required, got %zu", ws,
                workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return fail(IFA4_ERR_WORKSPACE, "backward: workspace must be 16-byte aligned");
  int* status = nullptr;
  if ((rc = device_status_ptr(&status))) return rc;

  ifa4::BackwardKernelArgs a{};
  a.rel = static_cast<const uint16_t*>(p->rel);
  a.out = static_cast<const uint16_t*>(p->out);
  a.dout = static_cast<const uint16_t*>(p->dout);
  a.lse = p->lse;
  a.delta = static_cast<float*>(workspace);
  a.dq = static_cast<uint16_t*>(p->dq);
  a.dk = static_cast<uint16_t*>(p->dk);
  a.dv = static_cast<uint16_t*>(p->dv);
  a.drel = static_cast<uint16_t*>(p->drel);
  a.cu_q = p->cu_seqlens_q;
  a.cu_k = p->cu_seqlens_k;
  a.rel_st = p->rel_stride_t;
  a.rel_sh = p->rel_stride_h;
  a.out_st = p->out_stride_t;
  a.out_sh = p->out_stride_h;
  a.dout_st = p->dout_stride_t;
  a.dout_sh = p->dout_stride_h;
  a.lse_sh = p->lse_stride_h;
  a.lse_st = p->lse_stride_t;
  a.dq_st = p->dq_stride_t;
  a.dq_sh = p->dq_stride_h;
  a.dk_st = p->dk_stride_t;
  a.dk_sh = p->dk_stride_h;
  a.dv_st = p->dv_stride_t;
  a.dv_sh = p->dv_stride_h;
  a.drel_st = p->drel_stride_t;
  a.drel_sh = p->drel_stride_h;
  a.total_q = p->total_q;
  a.total_k = p->total_k;
  a.batch = p->batch;
  a.n_heads = p->n_heads;
  a.kv_heads = p->kv_heads;
  a.rel_extent = p->rel_extent;
  a.causal = p->causal ? 1 : 0;
  a.window_left = p->window_left < 0 ? -1 : p->window_left;
  a.align_bottom_right = p->causal_align == IFA4_ALIGN_BOTTOM_RIGHT;
  a.scale = p->softmax_scale;
  a.scale_log2 = p->softmax_scale * 1.4426950408889634f;
  a.bias_vec = aligned16(p->rel) && p->rel_stride_t % 8 == 0 && p->rel_stride_h % 8 == 0 &&
               p->rel_extent % 8 == 0;
  // Grid orders (as in the forward): the slots of one head run together when the operand
  // stream of a tile over all heads (512 bytes per token and head: Q and dO for dK/dV, K and V
  // for dQ; average sequence, capped by the window) is more than a third of the L2.
  {
    int64_t span_q = (p->total_q + p->batch - 1) / p->batch;
    int64_t span_k = (p->total_k + p->batch - 1) / p->batch;
    if (p->window_left >= 0) {
      if (p->window_left + 256 < span_q) span_q = p->window_left + 256;
      if (p->window_left + 256 < span_k) span_k = p->window_left + 256;
    }
    a.slots_first_dkdv = span_q * p->n_heads * 512 > (48LL << 20);
    a.slots_first_dq = span_k * p->kv_heads * 512 > (48LL << 20);
  }
  a.status = status;

  CUtensorMap tq, tk, tv, tdo;
  const int64_t krows = p->total_k > 0 ? p->total_k : 1;
  if ((rc = encode_rows_heads_dims(&tq, p->q, p->total_q, p->n_heads, p->q_stride_t,
                                   p->q_stride_h, 128, "q")))
    return rc;
  if ((rc = encode_rows_heads_dims(&tdo, p->dout, p->total_q, p->n_heads, p->dout_stride_t,
                                   p->dout_stride_h, 128, "dout")))
    return rc;
  if ((rc = encode_rows_heads_dims(&tk, p->k, krows, p->kv_heads, p->k_stride_t, p->k_stride_h,
                                   128, "k")))
    return rc;
  if ((rc = encode_rows_heads_dims(&tv, p->v, krows, p->kv_heads, p->v_stride_t, p->v_stride_h,
                                   128, "v")))
    return rc;
  int64_t max_sq = p->max_seqlen_q > 0 ? p->max_seqlen_q : p->total_q;
  if (max_sq > p->total_q) max_sq = p->total_q;
  int64_t max_sk = p->max_seqlen_k > 0 ? p->max_seqlen_k : p->total_k;
  if (max_sk > p->total_k) max_sk = p->total_k;
  int64_t qs = (max_sq + 127) / 128, ks = (max_sk + 127) / 128;
  qs = qs < 1 ? 1 : (qs > 65535 ? 65535 : qs);
  ks = ks < 1 ? 1 : (ks > 65535 ? 65535 : ks);
  cudaError_t e = ifa4::launch_backward_sm100(a, tq, tk, tv, tdo, static_cast<int>(qs),
                                              static_cast<int>(ks),
                                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "backward launch");
  return IFA4_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// rel_logits producer
// ---------------------------------------------------------------------------------------
namespace {
int validate_rel_logits(const IFA4RelLogitsParams* p) {
  if (p == nullptr) return fail(IFA4_ERR_INVALID_ARGUMENT, "rel_logits: params is NULL");
  if (p->dtype != IFA4_DTYPE_BF16)
    return fail(IFA4_ERR_UNSUPPORTED, "rel_logits: dtype %d unsupported (bf16 only)", p->dtype);
  if (p->d_rel != 16)
    return fail(IFA4_ERR_UNSUPPORTED, "rel_logits: d_rel %d unsupported (16 only)", p->d_rel);
  if (p->total_q < 0 || p->n_heads <= 0 || p->rel_extent <= 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT,
                "rel_logits: total_q must be >= 0, n_heads and rel_extent > 0");
  if (p->rel_extent % 8 != 0)
    return fail(IFA4_ERR_UNSUPPORTED, "rel_logits: rel_extent %d is not a multiple of 8",
                p->rel_extent);
  if (p->total_q > 2147483647LL - 256)
    return fail(IFA4_ERR_UNSUPPORTED, "rel_logits: total_q beyond 2^31 - 256");
  if (static_cast<int64_t>(p->n_heads) * ((p->rel_extent + 127) / 128) > (1LL << 30))
    return fail(IFA4_ERR_UNSUPPORTED, "rel_logits: n_heads x rel_extent / 128 beyond 2^30");
  if (!(p->nf > 0.f) || !(p->nf < 3.0e38f) || !(p->alpha > -3.0e38f && p->alpha < 3.0e38f))
    return fail(IFA4_ERR_INVALID_ARGUMENT, "rel_logits: nf must be finite and > 0, alpha finite");
  if (p->cu_seqlens_k != nullptr && p->cu_seqlens_q == nullptr)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "rel_logits: cu_seqlens_k given without cu_seqlens_q");
  if (p->cu_seqlens_q != nullptr && p->batch <= 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "rel_logits: batch must be > 0 with cu_seqlens_q");
  if (p->total_q == 0) return IFA4_OK;
  if (!p->r || !p->weight || !p->rel)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "rel_logits: null tensor pointer");
  if (!aligned16(p->r) || !aligned16(p->rel))
    return fail(IFA4_ERR_INVALID_ARGUMENT, "rel_logits: r and rel must be 16-byte aligned");
  const int64_t s8[] = {p->r_stride_t, p->r_stride_h, p->rel_stride_t, p->rel_stride_h};
  for (int64_t s : s8)
    if (s <= 0 || (s % 8) != 0)
      return fail(IFA4_ERR_INVALID_ARGUMENT,
                  "rel_logits: r and rel token/head strides must be positive multiples of 8 "
                  "elements");
  if (!aligned16(p->weight) || p->weight_stride_h < 0 || p->weight_stride_j <= 0 ||
      p->weight_stride_h % 8 != 0 || p->weight_stride_j % 8 != 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT,
                "rel_logits: weight must be 16-byte aligned with head stride a multiple of 8 "
                "elements (0 = shared) and row stride a positive multiple of 8");
  return IFA4_OK;
}
}  // namespace

extern "C" {

int ifa4_rel_logits_launch(const IFA4RelLogitsParams* p, void* stream) {
  g_last_error[0] = '\0';
  int rc = validate_rel_logits(p);
  if (rc) return rc;
  if (p->total_q == 0) return IFA4_OK;
  int* status = nullptr;
  if ((rc = device_status_ptr(&status))) return rc;
  int sms = 0;
  if ((rc = sm_count(&sms))) return rc;

  EncodeTiledFn fn;
  if ((rc = get_encode_fn(&fn))) return rc;
  CUtensorMap trel;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(p->rel_extent),
                        static_cast<cuuint64_t>(p->n_heads), static_cast<cuuint64_t>(p->total_q)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(p->rel_stride_h) * 2,
                           static_cast<cuuint64_t>(p->rel_stride_t) * 2};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(&trel, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p->rel, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(IFA4_ERR_UNSUPPORTED,
                "cuTensorMapEncodeTiled(rel) failed with CUresult %d (total_q=%lld heads=%d "
                "rel_extent=%d stride_t=%lld stride_h=%lld)",
                static_cast<int>(r), static_cast<long long>(p->total_q), p->n_heads,
                p->rel_extent, static_cast<long long>(p->rel_stride_t),
                static_cast<long long>(p->rel_stride_h));

  ifa4::RelLogitsKernelArgs a{};
  a.r = static_cast<const uint16_t*>(p->r);
  a.w = static_cast<const uint16_t*>(p->weight);
  a.cu_q = p->cu_seqlens_q;
  a.cu_k = p->cu_seqlens_q != nullptr ? p->cu_seqlens_k : nullptr;
  a.r_st = p->r_stride_t;
  a.r_sh = p->r_stride_h;
  a.w_sh = p->weight_stride_h;
  a.w_sj = p->weight_stride_j;
  a.total_q = p->total_q;
  a.batch = p->cu_seqlens_q != nullptr ? p->batch : 1;
  a.n_heads = p->n_heads;
  a.rel_extent = p->rel_extent;
  a.col_blocks = (p->rel_extent + 127) / 128;
  a.head_quads = (p->n_heads + 3) / 4;
  a.units = ((p->total_q + 127) / 128) * static_cast<int64_t>(a.head_quads) * a.col_blocks;
  a.alpha = p->alpha;
  a.nf = p->nf;
  a.status = status;
  const int64_t cap = static_cast<int64_t>(sms) * ifa4::kRelLogitsCtasPerSm;
  const int grid = static_cast<int>(a.units < cap ? a.units : cap);
  cudaError_t e = ifa4::launch_rel_logits_sm100(a, trel, grid, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rel_logits launch");
  return IFA4_OK;
}

int ifa4_selftest_bounded_wait(int64_t timeout_ns, void* stream) {
  g_last_error[0] = '\0';
  if (timeout_ns <= 0 || timeout_ns > 1000000000LL)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "selftest: timeout_ns must be in (0, 1e9]");
  int* status = nullptr;
  int rc = device_status_ptr(&status);
  if (rc) return rc;
  ifa4_selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<unsigned long long>(timeout_ns));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return IFA4_OK;
}

int ifa4_measure_read_stream(const void* buf, size_t bytes, uint32_t* sink, void* stream) {
  g_last_error[0] = '\0';
  if (buf == nullptr || sink == nullptr || bytes == 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "read_stream: null buffer or sink, or zero bytes");
  if ((reinterpret_cast<uintptr_t>(buf) & 15u) != 0 || (bytes & 15u) != 0)
    return fail(IFA4_ERR_INVALID_ARGUMENT, "read_stream: buffer and size must be 16-byte aligned");
  int sms = 148;
  int rc = sm_count(&sms);
  if (rc) return rc;
  ifa4_read_stream_kernel<<<sms * 4, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(buf), static_cast<unsigned long long>(bytes / 16), sink);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "read_stream launch");
  return IFA4_OK;
}

int ifa4_read_device_status(void* stream, int32_t clear, int32_t* status_out) {
  g_last_error[0] = '\0';
  if (status_out == nullptr) return fail(IFA4_ERR_INVALID_ARGUMENT, "status_out is NULL");
  int* dptr = nullptr;
  int rc = device_status_ptr(&dptr);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, dptr, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (clear && host != 0) {
    e = cudaMemsetAsync(dptr, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "clear status");
  }
  *status_out = host;
  return IFA4_OK;
}

}  // extern "C"
