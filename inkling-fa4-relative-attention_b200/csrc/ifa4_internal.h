// Internal interface between the C ABI layer (ifa4_capi.cu) and the kernel translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace ifa4 {

constexpr int kHeadDim = 128;

// Raises a kernel's dynamic shared-memory limit on the current device, once per device (the
// limit is a per-device function attribute).  `done` is one flag per device ordinal; it is
// atomic, so host threads launching at the same time do not race on it (two first calls may
// both set the attribute, which is harmless: the value is the same).
template <typename K>
cudaError_t set_smem_limit_once(K kernel, uint32_t bytes, std::atomic<bool> (&done)[64]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!done[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(bytes));
    if (e != cudaSuccess) return e;
    done[dev].store(true, std::memory_order_release);
  }
  return cudaSuccess;
}

// Status bits written by kernels that abandoned a bounded wait.
constexpr int kStatusPrefillTimeout = 1;
constexpr int kStatusDecodeTimeout = 2;
constexpr int kStatusBackwardTimeout = 4;
constexpr int kStatusSelfTestTimeout = 8;   // ifa4_selftest_bounded_wait, warp 0
constexpr int kStatusSelfTestOwnTimeout = 16;  // ifa4_selftest_bounded_wait, warp 1 (must not be set)
constexpr int kStatusRelLogitsTimeout = 32;
constexpr int kStatusDebugBounds = 64;   // debug builds only: an index range check failed

// Index range checks of debug builds (compiled with -DIFA4_DEBUG, the library's stand-in for a
// bounds-checking sanitizer): a failed check ORs kStatusDebugBounds into the status word and the
// guarded access is skipped, so a bad index is reported without touching memory out of range.
// In release builds the condition is not evaluated and the access is unconditional.
#ifdef IFA4_DEBUG
__device__ __forceinline__ bool debug_check(int* status, bool ok) {
  if (!ok && status != nullptr) atomicOr(status, kStatusDebugBounds);
  return ok;
}
#define IFA4_DBG_CHECK(status, cond) ::ifa4::debug_check((status), (cond))
#else
#define IFA4_DBG_CHECK(status, cond) true
#endif

struct PrefillKernelArgs {
  const uint16_t* rel;       // bf16 bits
  uint16_t* out;             // bf16 bits
  const int32_t* cu_q;
  const int32_t* cu_k;
  long long rel_st, rel_sh;
  long long out_st, out_sh;
  int batch, n_heads, kv_heads, rel_extent;
  int causal, window_left, align_bottom_right;
  int bias_vec;              // rel 16-byte aligned (base, strides) and rel_extent % 8 == 0:
                             // each row loads its bias with 16-byte vectors
  int pair_heads;            // 1: the CTA's two sub-tiles are two heads at the same rows
                             // 0: the CTA's two sub-tiles are consecutive 128-row blocks
  int q_fastest;             // grid (query slots, head slots, sequences) rather than
                             // (head slots, sequences, query slots)
  float scale_log2;          // softmax_scale * log2(e)
  float* lse;                // optional natural-log LSE, [h * lse_sh + token * lse_st]
  long long lse_sh, lse_st;
  // paged KV cache (kernels instantiated with kPaged): K/V tensor maps are 4-D
  // {128 dims, kv_heads, page_size, num_pages}; tiles load in units of 2^box_shift rows
  const int32_t* block_table;
  long long bt_stride;
  int page_shift, box_shift, num_pages;
  const uint16_t* v;         // V cache base (partial last unit copied with plain loads)
  long long v_st, v_sh, v_sp;
  int* status;
  // output copies on other GPUs: element e of out is also stored at out + out_peer_delta[i] + e
  long long out_peer_delta[7];
  int n_out_peers;
  // KV split (kv_splits > 1): the query tile's KV tiles are cut into kv_splits ranges, one per
  // CTA; each writes its rows' normalised fp32 partial output and log2-sum-exp, and
  // rel_attn_prefill_combine_kernel merges them into out (and lse)
  int kv_splits;
  float* ws_o;               // [kv_splits, total_q, n_heads, 128]
  float* ws_lse;             // [kv_splits, n_heads, total_q], log2 units, -inf: no visible key
  long long total_q;
};

struct PrefillLaunch {
  dim3 grid;
  int smem_bytes;
};

// Prefill tile configurations: the kernel variants differ in where the exponentials of every 16
// score columns are computed: FMA-pipe polynomial, SFU two-at-a-time (f16x2), or SFU fp32.
// tile_config 0 = automatic (2 polynomial columns of 16); 1..5 = 0, 2, 4, 6, 8 polynomial columns of 16; 6 = all f16x2; 7 = 8 of 16 f16x2;
// 8 = 4 polynomial + 8 f16x2.
constexpr int kPrefillDefaultEmu = 2;
constexpr int kPrefillDefaultHalf2 = 0;
constexpr int kPrefillNumTileConfigs = 9;
int prefill_emulated_exp_columns(int tile_config);  // -1 for an unknown id

// Launches the tcgen05 prefill kernel variant of `tile_config`.  Returns a cudaError_t.
// With a paged cache (args.block_table != nullptr) only tile configs 0 to 3 exist.
cudaError_t launch_prefill_sm100(const PrefillKernelArgs& args, const CUtensorMap& tm_q,
                                 const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                 int q_slots, int tile_config, int max_seqlen_q,
                                 cudaStream_t stream);
// Merge of the kv_splits partials written by a split launch (one warp per token and head).
cudaError_t launch_prefill_combine_sm100(const PrefillKernelArgs& args, cudaStream_t stream);
bool prefill_paged_tile_config_ok(int tile_config);

struct DecodeKernelArgs {
  const uint16_t* q;
  const uint16_t* rel;
  uint16_t* out;
  const int32_t* cu_q;
  const int32_t* cu_k;
  long long q_st, q_sh;
  long long rel_st, rel_sh;
  long long out_st, out_sh;
  int batch, n_heads, kv_heads, rel_extent;
  int causal, window_left, align_bottom_right;
  int group;                 // n_heads / kv_heads
  int heads_per_cta;         // <= 16 query heads of one kv group per CTA
  int num_splits;            // CTAs per (sequence, head block)
  int chunk_len;             // keys per chunk (multiple of 64)
  float scale_log2;
  float* ws_o;               // [batch, n_heads, num_splits, 128] (num_splits > 1)
  float* ws_lse;             // [batch, n_heads, num_splits]      (num_splits > 1)
  float* lse;                // optional natural-log LSE output
  long long lse_sh, lse_st;
  const int32_t* block_table;  // paged KV cache, as in PrefillKernelArgs
  long long bt_stride;
  int page_shift, box_shift, num_pages;
  int* status;
};

cudaError_t launch_decode_sm100(const DecodeKernelArgs& args, const CUtensorMap& tm_k,
                                const CUtensorMap& tm_v, cudaStream_t stream);

struct BackwardKernelArgs {
  const uint16_t* rel;       // bf16 bits
  const uint16_t* out;       // forward output O
  const uint16_t* dout;      // incoming gradient dO
  const float* lse;          // forward natural-log LSE, [h * lse_sh + token * lse_st]
  float* delta;              // workspace [n_heads, total_q]: rowsum(dO * O)
  long long total_k;         // rows of k / v / dk / dv (index checks of debug builds)
  uint16_t* dq;
  uint16_t* dk;
  uint16_t* dv;
  uint16_t* drel;
  const int32_t* cu_q;
  const int32_t* cu_k;
  long long rel_st, rel_sh, out_st, out_sh, dout_st, dout_sh, lse_sh, lse_st;
  long long dq_st, dq_sh, dk_st, dk_sh, dv_st, dv_sh, drel_st, drel_sh;
  long long total_q;
  int batch, n_heads, kv_heads, rel_extent;
  int causal, window_left, align_bottom_right;
  float scale;               // softmax_scale
  float scale_log2;          // softmax_scale * log2(e)
  int bias_vec;              // rel 16-byte aligned and rel_extent % 8 == 0 (vector bias windows)
  int slots_first_dkdv;      // dK/dV grid (key slots, kv heads, sequences) instead of
                             // (kv heads, sequences, key slots)
  int slots_first_dq;        // dQ grid (query slots, heads, sequences) instead of
                             // (heads, sequences, query slots)
  int* status;
};

// rel_logits producer: rel[t, h, e] = bf16(tau(pos_t) * sum_j r[t, h, j] * W_h[j, e]).
struct RelLogitsKernelArgs {
  const uint16_t* r;         // bf16 bits, r[t * r_st + h * r_sh + j], j < 16
  const uint16_t* w;         // bf16 bits, W_h[j, e] at w[h * w_sh + j * w_sj + e]
  const int32_t* cu_q;       // optional (null: one sequence)
  const int32_t* cu_k;       // optional (null: positions start at 0)
  long long r_st, r_sh, w_sh, w_sj;
  long long total_q;
  long long units;           // quads: token tiles x head_quads x col_blocks
  int batch, n_heads, rel_extent;
  int head_quads;            // ceil(n_heads / 4)
  int col_blocks;            // ceil(rel_extent / 128)
  float alpha, nf;
  int* status;
};

// Grid of `grid` CTAs (up to kRelLogitsCtasPerSm per SM) striding over args.units quads of
// 128 tokens x 4 heads x 128 columns; rel written through tm_rel ({rel_extent, n_heads, total_q},
// 64 x 1 x 128 boxes, 128-byte swizzle).
cudaError_t launch_rel_logits_sm100(const RelLogitsKernelArgs& args, const CUtensorMap& tm_rel,
                                    int grid, cudaStream_t stream);
constexpr int kRelLogitsCtasPerSm = 4;

// Prep (Delta, zeroed d rel band), dK/dV (+ d rel) and dQ kernels, in that order on `stream`.
cudaError_t launch_backward_sm100(const BackwardKernelArgs& args, const CUtensorMap& tm_q,
                                  const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                  const CUtensorMap& tm_do, int q_slots, int k_slots,
                                  cudaStream_t stream);

}  // namespace ifa4
