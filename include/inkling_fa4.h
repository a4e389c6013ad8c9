/*
 * inkling_fa4 — C ABI of the B200 (sm_100a) relative-position-bias flash attention.
 *
 * Plain pointers, integers and floats only.  All tensor pointers are device pointers; the
 * integer strides are in ELEMENTS.  Every call is asynchronous on the given CUDA stream
 * (passed as an opaque pointer: a cudaStream_t, or NULL for the legacy default stream) and
 * performs no host<->device synchronisation, so it can be captured in a CUDA graph.
 * Every entry point returns 0 on success or a negative IFA4_ERR_* code; the message of the
 * last failure on the calling thread is available from ifa4_last_error_string().
 *
 * Lifetime: the library caches, per device, the device addresses of its own __device__
 * objects (the status word, the no-allocation decode scratch).  Those addresses belong to the
 * device's primary context, so the library must not be used across a cudaDeviceReset() (or
 * any other destruction of the primary context) in the same process: the cached addresses
 * would then point into a released context.
 *
 * Semantics follow the reference oracle ref_rel_attn (src/inkling_fa4/reference.py:4-39 of
 * KINGXD414/Inkling-FA4-Relative-Attention): scores = (q k^T) * scale; bias
 * rel[q, h, d] with d = q_pos + bias_shift - k_pos applied only when 0 <= d < rel_extent;
 * causal mask k_pos <= q_pos + mask_shift; window mask q_pos + mask_shift - k_pos <= window;
 * GQA kv head = h / (n_heads / kv_heads).  causal_align = IFA4_ALIGN_REFERENCE gives
 * mask_shift = 0, bias_shift = sq - sk (reference.py:28-37); IFA4_ALIGN_BOTTOM_RIGHT gives
 * mask_shift = bias_shift = sk - sq.  Rows with no visible key produce 0 (the reference's
 * Triton kernel behaviour, triton_kernel.py:65-67,79).
 */
#ifndef INKLING_FA4_H_
#define INKLING_FA4_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IFA4_ABI_VERSION 7

enum {
  IFA4_OK = 0,
  IFA4_ERR_INVALID_ARGUMENT = -1,  /* null pointer, bad shape/stride/alignment/value   */
  IFA4_ERR_UNSUPPORTED = -2,       /* valid input the kernels do not implement         */
  IFA4_ERR_CUDA = -3,              /* a CUDA runtime/driver call failed                 */
  IFA4_ERR_WORKSPACE = -4,         /* decode workspace missing or too small             */
  IFA4_ERR_DEVICE_TIMEOUT = -5     /* a kernel gave up on a bounded wait (status word)  */
};

enum { IFA4_ALIGN_REFERENCE = 0, IFA4_ALIGN_BOTTOM_RIGHT = 1 };
enum { IFA4_DTYPE_BF16 = 0 };

/* Varlen prefill / chunked prefill / sliding window.
 * q   [total_q, n_heads, head_dim]     k, v [total_k, kv_heads, head_dim]
 * rel [total_q, n_heads, >=rel_extent] (rel_stride_t may be 0: a per-head table)
 * out [total_q, n_heads, head_dim]     cu_seqlens_q/k int32 [batch + 1] on the device.
 * q/k/v strides and base addresses must be multiples of 16 bytes (TMA); the last dimension
 * of every tensor is contiguous.  head_dim must be 128. */
typedef struct IFA4PrefillParams {
  const void* q;
  const void* k;
  const void* v;
  const void* rel;
  void* out;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int64_t q_stride_t, q_stride_h;
  int64_t k_stride_t, k_stride_h;
  int64_t v_stride_t, v_stride_h;
  int64_t rel_stride_t, rel_stride_h;
  int64_t out_stride_t, out_stride_h;
  int64_t total_q;          /* rows of q / rel / out                                  */
  int64_t total_k;          /* rows of k / v                                          */
  int32_t batch;
  int32_t n_heads;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t rel_extent;
  int32_t causal;           /* 0 or 1                                                  */
  int32_t window_left;      /* < 0 disables the sliding window                        */
  int32_t causal_align;     /* IFA4_ALIGN_*                                            */
  int32_t max_seqlen_q;     /* grid-size hint; <= 0 means "use total_q". Correctness does
                               not depend on it (CTAs stride over the query tiles).    */
  int32_t dtype;            /* IFA4_DTYPE_BF16                                         */
  float softmax_scale;      /* > 0; the reference uses 1/head_dim                      */
  int32_t tile_config;      /* 0 = automatic; see ifa4_prefill_tile_config_name        */
  /* Optional fp32 log-sum-exp of each row's scaled+biased logits (natural log; -inf for a
   * row with no visible key), written at lse[h * lse_stride_h + token * lse_stride_t] when
   * lse != NULL.  Not in the reference; callers merge split attention with it. */
  float* lse;
  int64_t lse_stride_h, lse_stride_t;
  /* Optional paged KV cache, used when block_table != NULL.  Not in the reference (its
   * serving-stack caller keeps K/V in 16-token pages).  k and v then point to caches
   * [num_pages, page_size, kv_heads, head_dim] with element strides (k_stride_page,
   * k_stride_t, k_stride_h, 1) (likewise v), and key j of sequence b sits in page
   * block_table[b * block_table_stride + j / page_size], slot j % page_size.  Key counts
   * still come from cu_seqlens_k (cu_seqlens_k[b+1] - cu_seqlens_k[b]); total_k is ignored.
   * page_size is a power of two >= 16; page strides are positive multiples of 8 elements.
   * Each sequence's table row must hold ceil(keys / page_size) entries; an entry outside
   * [0, num_pages) reads as zero keys and values.  Cache slots past a sequence's last key are
   * never used, whatever they hold (NaN included). */
  const int32_t* block_table;
  int64_t block_table_stride;
  int64_t k_stride_page, v_stride_page;
  int32_t page_size;
  int32_t num_pages;
  /* Optional copies of the output on other GPUs (ABI version 6; not in the reference, whose
   * single-GPU call has no multi-GPU path).  When n_out_peers > 0, out_peers is a host array of
   * n_out_peers device addresses, valid in this process, each pointing at the element that
   * corresponds to out[0] in another buffer laid out exactly like the one out points into
   * (typically another GPU's output buffer mapped into this process by CUDA IPC).  The kernel
   * stores every output row to out and, at the same offset, to each of these buffers as its
   * tiles finish, so ranks that each compute some heads of one call assemble the whole output on
   * every GPU during the call, with no gather afterwards.  Plain 16-byte stores (no TMA, no
   * multicast); 16-byte aligned addresses; at most IFA4_MAX_OUT_PEERS.  The writes are complete
   * when the launch completes; the caller orders the other GPUs' reads after that (a barrier in
   * stream order) and keeps them from reading while a later call overwrites the buffers. */
  const void* const* out_peers;
  int32_t n_out_peers;
  /* KV split (ABI version 7; not in the reference).  With ifa4_prefill_launch_ws, 0 lets the
   * library split each query tile's KV tiles over up to IFA4_MAX_KV_SPLITS CTAs when the grid
   * would leave SMs idle (small batches, few heads), with a merge kernel combining the partials;
   * a value > 1 forces that many splits; 1 never splits.  ifa4_prefill_launch accepts only 0 or 1
   * (it has no workspace and never splits). */
  int32_t kv_splits;
  /* Longest key sequence, a hint (ABI version 7; <= 0: unknown).  Only the automatic KV-split
   * choice of ifa4_prefill_launch_ws reads it (the same value gives the same choice whatever the
   * K/V layout); correctness never depends on it. */
  int32_t max_seqlen_k;
} IFA4PrefillParams;

#define IFA4_MAX_OUT_PEERS 7
#define IFA4_MAX_KV_SPLITS 16

/* Prefill.  Replaces the per-sequence launch loop of inkling_fa4_rel_attention_triton
 * (src/inkling_fa4/triton_kernel.py:84-106) and of the KV-pruned variant
 * (src/inkling_fa4/triton_kernel_kv_pruned.py:210-279): one launch covers all sequences,
 * cu_seqlens are read on the device, and masked KV tiles are never loaded. */
int ifa4_prefill_launch(const IFA4PrefillParams* params, void* stream);

/* Bytes of device workspace ifa4_prefill_launch_ws needs for these parameters (0 when the launch
 * does not split the KV range).  No counterpart in the reference, whose prefill launches one
 * Triton grid per sequence (triton_kernel.py:94-106); it sizes the caller-owned workspace. */
int ifa4_prefill_workspace_size(const IFA4PrefillParams* params, size_t* bytes_out);

/* Prefill with a caller workspace, which lets small launches (a grid smaller than the GPU: few
 * sequences, few heads) split each query tile's KV range over several CTAs: each writes a
 * normalised fp32 partial and its log-sum-exp into the workspace ([splits, total_q, n_heads,
 * 128] then [splits, n_heads, total_q] floats) and a merge kernel writes out (and lse).  Same
 * parameters and results as ifa4_prefill_launch (within rounding: the partials are merged in
 * fp32).  Replaces, like ifa4_prefill_launch, the launch loop of inkling_fa4_rel_attention_triton
 * (src/inkling_fa4/triton_kernel.py:94-106).  The workspace must be 16-byte aligned and hold
 * ifa4_prefill_workspace_size bytes; it may be NULL when that size is 0. */
int ifa4_prefill_launch_ws(const IFA4PrefillParams* params, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Single-token decode (one query per sequence: q [batch, n_heads, head_dim], cu_seqlens_q
 * gives each query's row).  Split-KV: each sequence's visible key range is cut into chunks
 * of chunk_len keys processed by num_splits CTAs per (sequence, kv head); a combine kernel
 * merges the fp32 partials. */
typedef struct IFA4DecodeParams {
  const void* q;
  const void* k;
  const void* v;
  const void* rel;
  void* out;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int64_t q_stride_t, q_stride_h;
  int64_t k_stride_t, k_stride_h;
  int64_t v_stride_t, v_stride_h;
  int64_t rel_stride_t, rel_stride_h;
  int64_t out_stride_t, out_stride_h;
  int64_t total_q;
  int64_t total_k;
  int32_t batch;
  int32_t n_heads;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t rel_extent;
  int32_t causal;
  int32_t window_left;
  int32_t causal_align;
  int32_t max_seqlen_k;     /* split-size hint; <= 0 means "use total_k"             */
  int32_t dtype;
  float softmax_scale;
  int32_t num_splits;       /* 0 = automatic (from max_seqlen_k and the SM count)      */
  int32_t chunk_len;        /* 0 = automatic; otherwise a multiple of 64               */
  float* lse;               /* optional, as in IFA4PrefillParams (token = the query row) */
  int64_t lse_stride_h, lse_stride_t;
  /* optional paged KV cache, as in IFA4PrefillParams */
  const int32_t* block_table;
  int64_t block_table_stride;
  int64_t k_stride_page, v_stride_page;
  int32_t page_size;
  int32_t num_pages;
} IFA4DecodeParams;

/* Decode.  Replaces inkling_fa4_rel_attention_decode_triton
 * (src/inkling_fa4/triton_kernel_decode.py:127-170), with the semantics of the oracle
 * (reference.py:4-39) rather than of that kernel. */
int ifa4_decode_launch(const IFA4DecodeParams* params, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Bytes of device workspace ifa4_decode_launch needs for these parameters (0 when a single
 * split suffices).  Resolves num_splits/chunk_len exactly as the launch does; writes them to
 * *num_splits_out / *chunk_len_out when those are non-null.  No new counterpart in the
 * reference (its decode has no split-KV); it sizes the caller-owned workspace. */
int ifa4_decode_workspace_size(const IFA4DecodeParams* params, size_t* bytes_out,
                               int32_t* num_splits_out, int32_t* chunk_len_out);

/* Size of the library-owned decode scratch used by ifa4_decode_launch_noalloc (16 MiB). */
#define IFA4_NOALLOC_DECODE_SCRATCH_BYTES (16u * 1024u * 1024u)

/* Decode for callers that cannot allocate device memory.  No counterpart in the reference.
 *
 * Some callers may not call cudaMalloc: a serving engine that reserves all device memory up
 * front and forbids allocation on its request path, or a plugin reached through a C FFI that
 * has no handle on its host's allocator and so cannot hand ifa4_decode_launch a workspace.
 * This entry point takes no workspace and allocates nothing: the split-KV partials go to a
 * statically sized array inside the library (IFA4_NOALLOC_DECODE_SCRATCH_BYTES), which every
 * GPU that loads the library holds until the process exits.
 *
 * Same parameters and results as ifa4_decode_launch.  With num_splits = 0 the split count is
 * capped so the partials fit the array; an explicit num_splits whose partials would not fit
 * is rejected with IFA4_ERR_WORKSPACE.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  All calls share the one array: calls whose kernels overlap on
 * the GPU (different streams, or different host threads) race on it, so serialise them.
 * Nothing in the array needs to start at zero: every split writes its whole partial before
 * the combine kernel reads it. */
int ifa4_decode_launch_noalloc(const IFA4DecodeParams* params, void* stream);

/* Backward of the prefill (varlen, causal / window, both alignments, GQA): gradients of the
 * loss with respect to q, k, v and rel_logits given dout = dLoss/dout.  Not in the reference
 * (it has no backward); the gradients are those of its forward, reference.py:4-39.
 * out and lse are the forward's output and its log-sum-exp (IFA4PrefillParams.lse).
 * dq [total_q, n_heads, 128], dk / dv [total_k, kv_heads, 128] are written in full (rows of
 * keys no query sees get 0); drel [total_q, n_heads, >= rel_extent] has columns [0, rel_extent)
 * written (the band gradient, 0 elsewhere) and later columns left untouched.  dout, dq, dk, dv
 * and out follow q's layout rules (16-byte aligned, strides multiples of 8 elements); drel and
 * lse need only a contiguous last dimension.  Deterministic: no atomics. */
typedef struct IFA4BackwardParams {
  const void* q;
  const void* k;
  const void* v;
  const void* rel;
  const void* out;
  const void* dout;
  const float* lse;
  void* dq;
  void* dk;
  void* dv;
  void* drel;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int64_t q_stride_t, q_stride_h;
  int64_t k_stride_t, k_stride_h;
  int64_t v_stride_t, v_stride_h;
  int64_t rel_stride_t, rel_stride_h;
  int64_t out_stride_t, out_stride_h;
  int64_t dout_stride_t, dout_stride_h;
  int64_t lse_stride_h, lse_stride_t;
  int64_t dq_stride_t, dq_stride_h;
  int64_t dk_stride_t, dk_stride_h;
  int64_t dv_stride_t, dv_stride_h;
  int64_t drel_stride_t, drel_stride_h;
  int64_t total_q;
  int64_t total_k;
  int32_t batch;
  int32_t n_heads;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t rel_extent;
  int32_t causal;
  int32_t window_left;
  int32_t causal_align;
  int32_t max_seqlen_q;     /* grid-size hints, as in IFA4PrefillParams                 */
  int32_t max_seqlen_k;
  int32_t dtype;
  float softmax_scale;
} IFA4BackwardParams;

/* Device workspace (bytes, 16-byte aligned) ifa4_backward_launch needs: fp32 row statistics. */
int ifa4_backward_workspace_size(const IFA4BackwardParams* params, size_t* bytes_out);

/* Backward.  Three kernels in order on `stream`: row statistics (and zeroing of the drel
 * band), dK / dV / drel per key block, dQ per query tile. */
int ifa4_backward_launch(const IFA4BackwardParams* params, void* workspace,
                         size_t workspace_bytes, void* stream);

/* rel_logits producer: the step before the attention in the Inkling layer (RelLogitsProj plus
 * the log-tau scaling, outputs/architecture.md:51-64 of the reference repository, which holds
 * only that diagram and no code for it), fused into one kernel:
 *   rel[t, h, e] = bf16( tau(pos_t) * sum_{j < 16} r[t, h, j] * W_h[j, e] ),  0 <= e < rel_extent
 *   tau(p) = 1 + alpha * log(max((p + 1) / nf, 1))        (alpha = 0: tau = 1 exactly)
 * with fp32 products and sums (tensor cores) and one rounding to bf16.  pos_t is the token's
 * position in its sequence: t - cu_seqlens_q[b] for the sequence b holding t, plus
 * (len_k(b) - len_q(b)) when cu_seqlens_k is given (queries are the last len_q of len_k
 * positions, as in chunked prefill and decode).  cu_seqlens_q NULL means one sequence.
 * r    [total_q, n_heads, 16] bf16: 16-byte aligned base, strides multiples of 8 elements
 *      (a slice of a merged projection output qualifies).
 * W    [16, rel_extent] shared by all heads (weight_stride_h = 0) or [n_heads, 16, rel_extent]
 *      bf16: 16-byte aligned, last dimension contiguous, strides multiples of 8 elements.
 * rel  [total_q, n_heads, >= rel_extent] bf16: 16-byte aligned, strides multiples of 8
 *      elements; columns [0, rel_extent) written.  rel_extent must be a multiple of 8.
 * The kernel's one wait per tile is bounded like the others (status bit 5). */
typedef struct IFA4RelLogitsParams {
  const void* r;
  const void* weight;
  void* rel;
  const int32_t* cu_seqlens_q;  /* optional, int32 [batch + 1] on the device */
  const int32_t* cu_seqlens_k;  /* optional, int32 [batch + 1] on the device */
  int64_t r_stride_t, r_stride_h;
  int64_t weight_stride_h, weight_stride_j;
  int64_t rel_stride_t, rel_stride_h;
  int64_t total_q;
  int32_t batch;      /* number of sequences (1 when cu_seqlens_q is NULL) */
  int32_t n_heads;
  int32_t d_rel;      /* must be 16 */
  int32_t rel_extent;
  int32_t dtype;
  float alpha;
  float nf;           /* > 0 */
} IFA4RelLogitsParams;

int ifa4_rel_logits_launch(const IFA4RelLogitsParams* params, void* stream);

/* Self-test of the failure detection (test hook; the reference has no counterpart): launches
 * on `stream` a kernel whose barrier wait can never complete, so the kernels' bounded-wait path
 * runs out after timeout_ns (0 < timeout_ns <= 1e9).  Afterwards the status word holds exactly
 * bit 3 (value 8): one waiter timed out and the other left through the abort flag it raised
 * (bit 4 would mean the abort did not propagate).  Nothing faults; the context stays usable.
 * Run it alone: while the status word is nonzero, concurrently running kernels of this library
 * abandon their waits too (that is how one failure stops the others). */
int ifa4_selftest_bounded_wait(int64_t timeout_ns, void* stream);

/* Measurement hook (no counterpart in the reference): launches on `stream` one read-only pass
 * over `bytes` bytes at `buf` (16-byte aligned, bytes a multiple of 16) with 16-byte
 * non-coherent loads, four in flight per thread, 4 CTAs of 512 threads per SM.  Timing it gives
 * the HBM read-stream ceiling against which the decode kernel (about 99 % reads) is judged.
 * `sink` is a device word that is written only in the unlikely event that the folded data
 * equal a fixed constant. */
int ifa4_measure_read_stream(const void* buf, size_t bytes, uint32_t* sink, void* stream);

/* Reads (and optionally clears) the library's device status word on `stream`, blocking the
 * calling thread until the stream has reached this point.  Nonzero means a kernel gave up on
 * a bounded wait (a bug, never expected): bit 0 prefill, bit 1 decode, bit 2 backward, bits 3-4
 * ifa4_selftest_bounded_wait, bit 5 rel_logits producer, bit 6 (debug builds compiled with
 * -DIFA4_DEBUG only) an index range check failed and the access was skipped.  Test hook; the
 * reference has no counterpart. */
int ifa4_read_device_status(void* stream, int32_t clear, int32_t* status_out);

/* Name of the sm_100a prefill tile configuration `tile_config` resolves to (the counterpart
 * of autotune_configs.get_preset, src/inkling_fa4/autotune_configs.py:61-85). */
const char* ifa4_prefill_tile_config_name(int32_t tile_config);

/* Message of the last error on the calling thread ("" if none). */
const char* ifa4_last_error_string(void);

/* IFA4_ABI_VERSION of the loaded library. */
int32_t ifa4_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* INKLING_FA4_H_ */
