// Backward pass of the relative-bias attention for sm_100a (B200): dQ, dK, dV and the gradient
// of the relative logits.  The reference has no backward; the gradients are those of its
// forward (reference.py:4-39) as torch autograd computes them through the oracle.
//
// With P = softmax(S * scale + bias) (masked), O = P V, L = logsumexp row statistic saved by the
// forward (natural log) and dO the incoming gradient:
//   Delta_i = sum_d dO_id O_id                        (prep kernel)
//   dP = dO V^T,  dS = P o (dP - Delta)                (dS = gradient of the biased logits)
//   dV = P^T dO,  dK = scale dS^T Q,  dQ = scale dS K,  d rel[i, h, d] = dS_ij for the key j at
//   bias distance d = q_pos + bias_shift - k_pos (each (i, d) pair names one key, so the bias
//   gradient is a scatter of dS along the band, without atomics).
//
// Three launches on the caller's stream:
//   rel_attn_bwd_prep_kernel   Delta (fp32 workspace) and zeroes the band columns [0, R) of
//                              d rel; one warp per (token, head).  HBM bound.
//   rel_attn_bwd_dkdv_kernel   one CTA per (kv head, 128-key block): K and V stay in shared
//                              memory while the Q and dO tiles of every query head of the GQA
//                              group stream through a two-stage TMA ring.  The tensor core
//                              computes S^T = K Q^T and dP^T = V dO^T into TMEM with the keys on
//                              the 128 lanes, so P^T and dS^T are written back to TMEM as bf16
//                              and feed dV += P^T dO and dK += dS^T Q directly (A operand from
//                              TMEM, dO / Q as MN-major B operands): no shared-memory round
//                              trip and both accumulators stay in TMEM (S^T | dP^T | dV | dK =
//                              512 columns).  The d rel band is scattered from dS^T here.
//   rel_attn_bwd_dq_kernel     one CTA per (query head, 128-row tile), shaped like the
//                              forward: Q and dO stay in shared memory, K / V stream; S = Q K^T
//                              is double-buffered in TMEM (S0 | S1 | dP | dQ) so the next tile's
//                              QK^T overlaps this tile's elementwise work; dQ += dS K with dS
//                              from TMEM.
// dK / dV / dQ are written once per CTA (no atomics), so the backward is deterministic.
//
// Warp roles in both tensor-core kernels (320 threads): warp 0 TMA producer, warp 1 UMMA issuer (one thread) and TMEM owner,
// warps 2-9 elementwise: warp w handles TMEM lanes 32 (w % 4) .. +31 (one row each) and columns
// 64 ((w - 2) / 4) .. +63 of the 128-column tile.
// There is no row reduction in the backward, so splitting columns between warps is free.
// All waits are bounded (status word on timeout), as in the forward kernels.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ifa4_internal.h"
#include "ifa4_ptx.cuh"

namespace ifa4 {
namespace bwd {

constexpr int kBM = 128;  // query rows per tile
constexpr int kBN = 128;  // keys per tile
constexpr int kThreads = 320;
constexpr uint32_t kHalf = 128u * 128u;  // 128 rows x 128 B (64 dims)
constexpr uint32_t kTile = 2u * kHalf;   // 128 rows x 256 B (128 dims)
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kIdescKM = idesc_bf16_f32(128, 128, /*b_mn_major=*/false);
constexpr uint32_t kIdescMN = idesc_bf16_f32(128, 128, /*b_mn_major=*/true);

// D[128 x 128] = A B^T over 128 dims, A and B K-major 128-row tiles (two swizzled halves).
__device__ __forceinline__ void mma_kk(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr) {
  const uint64_t ad = sdesc_sw128(a_addr, 16, 1024);
  const uint64_t bd = sdesc_sw128(b_addr, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
    umma_ss(d_tmem, sdesc_advance(ad, off), sdesc_advance(bd, off), kIdescKM, kk > 0 ? 1u : 0u);
  }
}

// D[128 x 128] (+)= A B with A in TMEM as bf16 (K = 128 split into two 64-wide halves stored
// at column offsets 0 and 64 of a_tmem, 32 columns each) and B a 128-row MN-major tile (rows
// = K, 128 dims = N).
__device__ __forceinline__ void mma_tk(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_addr,
                                       bool accumulate) {
  const uint64_t bd = sdesc_sw128(b_addr, kHalf, 1024);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ts(d_tmem, a_tmem + (kk >> 2) * 64 + (kk & 3) * 8, sdesc_advance(bd, kk * 2048),
            kIdescMN, (kk > 0 || accumulate) ? 1u : 0u);
}

__device__ __forceinline__ void store_row64_bf16(uint16_t* dst, const float* v, float mul) {
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * g + 0] * mul, v[8 * g + 1] * mul);
    w.y = pack_bf16x2(v[8 * g + 2] * mul, v[8 * g + 3] * mul);
    w.z = pack_bf16x2(v[8 * g + 4] * mul, v[8 * g + 5] * mul);
    w.w = pack_bf16x2(v[8 * g + 6] * mul, v[8 * g + 7] * mul);
    reinterpret_cast<uint4*>(dst)[g] = w;
  }
}

__device__ __forceinline__ void store_zero_row64(uint16_t* dst) {
#pragma unroll
  for (int g = 0; g < 8; ++g) reinterpret_cast<uint4*>(dst)[g] = make_uint4(0u, 0u, 0u, 0u);
}

// --------------------------------------------------------------------------------------
// prep: Delta[h, t] = <dO[t, h], O[t, h]> and d rel[t, h, 0:R) = 0
// --------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rel_attn_bwd_prep_kernel(const __grid_constant__
                                                                    BackwardKernelArgs a) {
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.total_q * a.n_heads) return;
  const long long t = row / a.n_heads;
  const int h = static_cast<int>(row % a.n_heads);
  const uint2 o = *reinterpret_cast<const uint2*>(a.out + t * a.out_st + h * a.out_sh + lane * 4);
  const uint2 g = *reinterpret_cast<const uint2*>(a.dout + t * a.dout_st + h * a.dout_sh + lane * 4);
  float acc = bf16_bits_to_float(o.x & 0xffffu) * bf16_bits_to_float(g.x & 0xffffu) +
              bf16_bits_to_float(o.x >> 16) * bf16_bits_to_float(g.x >> 16) +
              bf16_bits_to_float(o.y & 0xffffu) * bf16_bits_to_float(g.y & 0xffffu) +
              bf16_bits_to_float(o.y >> 16) * bf16_bits_to_float(g.y >> 16);
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  if (lane == 0) a.delta[static_cast<long long>(h) * a.total_q + t] = acc;
  uint16_t* dr = a.drel + t * a.drel_st + h * a.drel_sh;
  for (int d = lane; d < a.rel_extent; d += 32) dr[d] = 0;
}

// --------------------------------------------------------------------------------------
// dK / dV (and d rel)
// --------------------------------------------------------------------------------------
namespace kv {
constexpr uint32_t kSmemK = 0;
constexpr uint32_t kSmemV = kTile;
constexpr uint32_t kSmemQ = 2 * kTile;   // 2 stages
constexpr uint32_t kSmemDO = 4 * kTile;  // 2 stages
constexpr uint32_t kSmemBar = 6 * kTile;
// per elementwise warp, two buffers of -lse (log2 domain) and Delta of its 64 query columns
constexpr uint32_t kSmemVec = kSmemBar + 256;
// per elementwise warp, the relative-bias segments of 32 of its columns in a band step: five
// aligned 16-byte vectors (80 bytes) around the 32 distances its keys read in each column
constexpr uint32_t kStageColBytes = 80;
constexpr uint32_t kStageWarpBytes = 32 * kStageColBytes;
constexpr uint32_t kSmemStage = kSmemVec + 8 * 256 * 4;
constexpr uint32_t kSmemBytes = kSmemStage + 8 * kStageWarpBytes;
static_assert(kSmemBytes + 1024 <= 227u * 1024u, "dK/dV shared memory");
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384;

struct Bars {
  uint64_t kv_full, kv_empty;
  uint64_t qdo_full[2], qdo_empty[2];
  uint64_t s_full, dp_full, p_full, ds_full;
  uint64_t acc_full, acc_empty;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");
}  // namespace kv

// Query tiles a key block [k0, k0 + 128) contributes to: [i_lo, i_lo + n_q) (per head).
struct KeyBlock {
  int i_lo, n_q;
};

__device__ __forceinline__ KeyBlock key_block(const BackwardKernelArgs& a, int k0, int sq, int sk) {
  KeyBlock kb{0, 0};
  const int ms = a.align_bottom_right ? sk - sq : 0;
  const int k1 = min(k0 + kBN, sk);
  int lo = 0, hi = sq;
  if (a.causal) lo = max(0, k0 - ms);                         // q + ms >= k
  if (a.window_left >= 0) hi = min(hi, k1 - 1 - ms + a.window_left + 1);  // q + ms - k <= W
  if (k1 > k0 && hi > lo) {
    kb.i_lo = lo / kBM;
    kb.n_q = (hi + kBM - 1) / kBM - kb.i_lo;
  }
  return kb;
}

__global__ void __launch_bounds__(kThreads, 1)
    rel_attn_bwd_dkdv_kernel(const __grid_constant__ BackwardKernelArgs a,
                             const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v,
                             const __grid_constant__ CUtensorMap tm_do) {
  using namespace kv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kSmemBar);
  float* vec = reinterpret_cast<float*>(smem + kSmemVec);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid (key slots, kv heads, sequences) when the Q / dO stream over all heads outgrows L2
  // (the key blocks of one kv head then run together and share their Q / dO tiles in L2),
  // otherwise (kv heads, sequences, key slots).
  const int kvh = a.slots_first_dkdv ? blockIdx.y : blockIdx.x;
  const int b = a.slots_first_dkdv ? blockIdx.z : blockIdx.y;
  const int kb0 = a.slots_first_dkdv ? blockIdx.x : blockIdx.z;
  const int kb_step = a.slots_first_dkdv ? gridDim.x : gridDim.z;
  const int group = a.n_heads / a.kv_heads;
  const int q_start = a.cu_q[b];
  const int sq = a.cu_q[b + 1] - q_start;
  const int k_start = a.cu_k[b];
  const int sk = a.cu_k[b + 1] - k_start;
  const int n_kb = (sk + kBN - 1) / kBN;
  if (kb0 >= n_kb) return;  // uniform over the CTA

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    mbar_init(&bars->kv_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->qdo_full[i], 1);
      mbar_init(&bars->qdo_empty[i], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->p_full, 8);
    mbar_init(&bars->ds_full, 8);
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 8);
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const AbortCtx ab{&bars->abort_flag, a.status, kStatusBackwardTimeout};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t ic = 0, sc = 0;
      const uint64_t pol_kv = l2_policy_evict_first();
      const uint64_t pol_q = l2_policy_evict_last();
      bool ok = true;
      for (int kb = kb0; kb < n_kb && ok; kb += kb_step) {
        const KeyBlock blk = key_block(a, kb * kBN, sq, sk);
        if (blk.n_q == 0) continue;
        if (!(ok = mbar_wait(&bars->kv_empty, (ic & 1) ^ 1, ab))) break;
        mbar_arrive_expect_tx(&bars->kv_full, 2 * kTile);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_3d_hint(smem + kSmemK + hf * kHalf, &tm_k, &bars->kv_full, hf * 64, kvh,
                           k_start + kb * kBN, pol_kv);
          tma_load_3d_hint(smem + kSmemV + hf * kHalf, &tm_v, &bars->kv_full, hf * 64, kvh,
                           k_start + kb * kBN, pol_kv);
        }
        ++ic;
        for (int g = 0; g < group && ok; ++g) {
          const int h = kvh * group + g;
          for (int i = 0; i < blk.n_q; ++i, ++sc) {
            const uint32_t st = sc & 1;
            if (!(ok = mbar_wait(&bars->qdo_empty[st], ((sc >> 1) & 1) ^ 1, ab))) break;
            mbar_arrive_expect_tx(&bars->qdo_full[st], 2 * kTile);
            const int row = q_start + (blk.i_lo + i) * kBM;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              tma_load_3d_hint(smem + kSmemQ + st * kTile + hf * kHalf, &tm_q,
                               &bars->qdo_full[st], hf * 64, h, row, pol_q);
              tma_load_3d_hint(smem + kSmemDO + st * kTile + hf * kHalf, &tm_do,
                               &bars->qdo_full[st], hf * 64, h, row, pol_q);
            }
          }
        }
      }
      // drain: the loads of the last uses of every buffer have landed
      if (ic > 0) mbar_wait(&bars->kv_full, (ic - 1) & 1, ab);
      for (uint32_t i = 0; i < 2 && i < sc; ++i) {
        const uint32_t last = sc - 1 - i;
        mbar_wait(&bars->qdo_full[last & 1], (last >> 1) & 1, ab);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      uint32_t ic = 0, sc = 0;
      const uint32_t k_addr = smem_u32(smem + kSmemK);
      const uint32_t v_addr = smem_u32(smem + kSmemV);
      const uint32_t q_addr = smem_u32(smem + kSmemQ);
      const uint32_t do_addr = smem_u32(smem + kSmemDO);
      bool ok = true;
      for (int kb = kb0; kb < n_kb && ok; kb += kb_step) {
        const KeyBlock blk = key_block(a, kb * kBN, sq, sk);
        if (blk.n_q == 0) continue;
        if (!(ok = mbar_wait(&bars->kv_full, ic & 1, ab))) break;
        const int steps = group * blk.n_q;
        // Issue order per step n: dV(n) once P^T(n) is in TMEM; then, once dS^T(n) is, the
        // next step's S^T(n+1) (its region's last readers, the dS phase and dV(n), are done or
        // queued before it) ahead of dK(n) and dP^T(n+1), so the elementwise warps' P phase of
        // step n+1 runs while the tensor core computes dK(n) and dP^T(n+1).
        {
          const uint32_t st = sc & 1;
          if (!(ok = mbar_wait(&bars->qdo_full[st], (sc >> 1) & 1, ab))) break;
          tc_fence_after();
          mma_kk(tbase + kColS, k_addr, q_addr + st * kTile);    // S^T = K Q^T
          umma_commit(&bars->s_full);
          mma_kk(tbase + kColDP, v_addr, do_addr + st * kTile);  // dP^T = V dO^T
          umma_commit(&bars->dp_full);
        }
        for (int n = 0; n < steps; ++n, ++sc) {
          const uint32_t st = sc & 1;
          if (n == 0 && !(ok = mbar_wait(&bars->acc_empty, (ic & 1) ^ 1, ab))) break;
          if (!(ok = mbar_wait(&bars->p_full, sc & 1, ab))) break;
          tc_fence_after();
          mma_tk(tbase + kColDV, tbase + kColS, do_addr + st * kTile, n > 0);  // dV += P^T dO
          if (!(ok = mbar_wait(&bars->ds_full, sc & 1, ab))) break;
          const bool next = n + 1 < steps;
          const uint32_t sn = (sc + 1) & 1;
          if (next && !(ok = mbar_wait(&bars->qdo_full[sn], ((sc + 1) >> 1) & 1, ab))) break;
          tc_fence_after();
          if (next) {
            mma_kk(tbase + kColS, k_addr, q_addr + sn * kTile);  // S^T(n+1)
            umma_commit(&bars->s_full);
          }
          mma_tk(tbase + kColDK, tbase + kColDP, q_addr + st * kTile, n > 0);  // dK += dS^T Q
          umma_commit(&bars->qdo_empty[st]);
          if (next) {
            mma_kk(tbase + kColDP, v_addr, do_addr + sn * kTile);  // dP^T(n+1)
            umma_commit(&bars->dp_full);
          }
        }
        if (!ok) break;
        umma_commit(&bars->acc_full);
        umma_commit(&bars->kv_empty);
        ++ic;
      }
      umma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, ab);
    }
  } else {
    // ------------------------------------------------------------------ elementwise + epilogue
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;        // columns [64 half, 64 half + 64)
    const int r = quarter * 32 + lane;       // key row within the block
    float* wvec = vec + (warp - 2) * 256;    // this warp's [2 buffers][-lse2 64 | Delta 64]
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tbase + lane_off + kColS + half * 64;
    const uint32_t t_dp = tbase + lane_off + kColDP + half * 64;
    const int ms = a.align_bottom_right ? sk - sq : 0;
    const int bs = a.align_bottom_right ? sk - sq : sq - sk;
    // Column statistics of step (head h, query tile q0) for this warp's 64 columns: lane holds
    // entries lane and lane + 32 of -lse (log2 domain) and of Delta.
    auto load_stats = [&](int h, int q0, float (&v)[4]) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int qq = q0 + half * 64 + ((lane + 32 * k) & 63);
        v[k] = 0.f;
        if (qq < sq) {
          const long long tok = q_start + qq;
          v[k] = k < 2 ? -a.lse[static_cast<long long>(h) * a.lse_sh + tok * a.lse_st] * kLog2e
                       : a.delta[static_cast<long long>(h) * a.total_q + tok];
        }
      }
    };
    auto store_stats = [&](uint32_t buf, const float (&v)[4]) {
#pragma unroll
      for (int k = 0; k < 4; ++k) wvec[buf * 128 + lane + 32 * k] = v[k];
    };
    uint32_t sc = 0, ec = 0;
    bool ok = true;
    for (int kb = kb0; kb < n_kb && ok; kb += kb_step) {
      const int k0 = kb * kBN;
      const KeyBlock blk = key_block(a, k0, sq, sk);
      const int kl = k0 + r;  // this thread's key (local to the sequence)
      const bool key_valid = kl < sk;
      IFA4_DBG_CHECK(a.status, !key_valid || k_start + kl < a.total_k);  // report only
      uint16_t* dk_row = a.dk + static_cast<long long>(k_start + kl) * a.dk_st +
                         static_cast<long long>(kvh) * a.dk_sh + half * 64;
      uint16_t* dv_row = a.dv + static_cast<long long>(k_start + kl) * a.dv_st +
                         static_cast<long long>(kvh) * a.dv_sh + half * 64;
      if (blk.n_q == 0) {  // no query sees these keys
        if (key_valid) {
          store_zero_row64(dk_row);
          store_zero_row64(dv_row);
        }
        continue;
      }
      const int steps = group * blk.n_q;  // (head g, query tile i) with i fastest
      {
        float v[4];
        load_stats(kvh * group, blk.i_lo * kBM, v);
        __syncwarp();
        store_stats(sc & 1, v);
      }
      for (int n = 0; n < steps; ++n, ++sc) {
        const int g = n / blk.n_q;
        const int h = kvh * group + g;
        const int q0 = (blk.i_lo + n - g * blk.n_q) * kBM;
        __syncwarp();  // this step's statistics are in wvec[sc & 1]
        const float* nl = wvec + (sc & 1) * 128;  // -lse2 of the 64 columns
        const float* dl = nl + 64;                // Delta
        // visible columns of this key: q in [c_lo, c_hi) relative to q0
        int c_lo = a.causal ? kl - ms - q0 : -0x40000000;
        int c_hi = sq - q0;
        if (a.window_left >= 0) c_hi = min(c_hi, kl - ms + a.window_left - q0 + 1);
        if (!key_valid) c_hi = -0x40000000;
        const bool has_mask = c_lo > half * 64 || c_hi < half * 64 + 64;
        // bias distance of column c (absolute 0..127): dq0 + c
        const int dq0 = q0 + bs - kl;
        const bool has_bias = key_valid && dq0 + half * 64 <= a.rel_extent - 1 &&
                              dq0 + half * 64 + 63 >= 0;
        const bool warp_bias = __any_sync(0xffffffffu, has_bias);
        const bool warp_slow = __any_sync(0xffffffffu, has_mask);  // bias: folded into nlr
        // The bias of a band step is read one value per (key, query) pair: for each of the 64
        // columns the warp's 32 keys read 32 consecutive distances (64 bytes) of that query's
        // rel row, a different row per column.  Those lines are pulled into L2 one step ahead,
        // so the step's loads wait on L2 rather than on DRAM: lane l takes columns l and l + 32,
        // at the distances of the warp's first and last key (in bounds by construction).
        if (n + 1 < steps) {
          const int g1 = (n + 1) / blk.n_q;
          const int q1 = (blk.i_lo + n + 1 - g1 * blk.n_q) * kBM;
          const int kl0 = k0 + quarter * 32;            // the warp's first key
          const int d_hi0 = q1 + bs - kl0 + half * 64;  // distance of (first key, column 0)
          const int d_lo0 = d_hi0 - 31;                 // (last key, column 0)
          if (d_lo0 <= a.rel_extent - 1 && d_hi0 + 63 >= 0) {  // some pair is in the band
            const uint16_t* rel_h1 = a.rel + static_cast<long long>(kvh * group + g1) * a.rel_sh;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int c = lane + 32 * k;
              const int qq = q1 + half * 64 + c;
              const int lo = max(d_lo0 + c, 0), hi = min(d_hi0 + c, a.rel_extent - 1);
              if (qq < sq && lo <= hi) {
                const uint16_t* row = rel_h1 + static_cast<long long>(q_start + qq) * a.rel_st;
                prefetch_l2(row + lo);
                prefetch_l2(row + hi);
              }
            }
          }
        }
        // -lse2 of the 64 columns into registers while S^T is computed: during the P phase the
        // tensor core streams dK / dP^T operands out of shared memory, and column loads issued
        // then stall the exponentials behind them
        float nlr[64];
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          const float4 L = *reinterpret_cast<const float4*>(nl + c);
          nlr[c] = L.x;
          nlr[c + 1] = L.y;
          nlr[c + 2] = L.z;
          nlr[c + 3] = L.w;
        }
        // Band step: the bias joins the exponent's per-column term, log2(e) * rel - lse2, here,
        // before the wait for S^T, so the loads' round trips overlap the S^T product rather than
        // the P phase (16 loads in flight at a time).
        if (warp_bias && a.bias_vec) {
          // The warp's 32 keys read, in column c, the 32 distances [dh + c - 31, dh + c] of that
          // query's rel row.  Per half of the columns the 32 segments go to shared memory as
          // five aligned 16-byte vectors each (cp.async: no registers held while in flight;
          // vectors outside [0, R) or past the sequence are not copied and not read), then each
          // lane reads its own 32 values: one round trip per half.
          const uint16_t* rel_h = a.rel + static_cast<long long>(h) * a.rel_sh;
          const int dh = q0 + bs - (k0 + quarter * 32) + half * 64;
          const uint8_t* stg = smem + kv::kSmemStage + (warp - 2) * kv::kStageWarpBytes;
          const uint32_t stg_s = smem_u32(stg);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
            for (int m = 0; m < 5; ++m) {
              const int t = lane + 32 * m;  // vector t of 160: column j, vector v
              const int j = t / 5, v = t - 5 * j;
              const int qq = q0 + half * 64 + hh * 32 + j;
              const int st = ((dh + hh * 32 + j - 31) & ~7) + 8 * v;
              if (qq < sq && st >= 0 && st < a.rel_extent &&
                  IFA4_DBG_CHECK(a.status, q_start + qq < a.total_q))
                cp_async16(stg_s + j * kv::kStageColBytes + v * 16,
                           rel_h + static_cast<long long>(q_start + qq) * a.rel_st + st);
            }
            cp_async_wait_all();
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int c = hh * 32 + i;
              const int cq = half * 64 + c;
              const int d = dq0 + cq;  // = dh + c - (this lane's key offset in the warp)
              float b = 0.f;
              if (has_bias && d >= 0 && d < a.rel_extent && cq < sq - q0) {
                const int base = (dh + c - 31) & ~7;
                b = bf16_bits_to_float(*reinterpret_cast<const uint16_t*>(
                    stg + i * kv::kStageColBytes + (d - base) * 2));
              }
              nlr[c] = fmaf(b, kLog2e, nlr[c]);
            }
            __syncwarp();  // every lane has read the stage before the next half overwrites it
          }
        } else if (warp_bias) {  // unaligned or odd-extent bias tensor: one load per value
          const uint16_t* rel_h = a.rel + static_cast<long long>(h) * a.rel_sh;
#pragma unroll
          for (int c16 = 0; c16 < 64; c16 += 16) {
            float b[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int cq = half * 64 + c16 + i;
              const int d = dq0 + cq;
              b[i] = 0.f;
              if (has_bias && d >= 0 && d < a.rel_extent && cq < sq - q0)
                b[i] = bf16_bits_to_float(
                    __ldg(rel_h + static_cast<long long>(q_start + q0 + cq) * a.rel_st + d));
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) nlr[c16 + i] = fmaf(b[i], kLog2e, nlr[c16 + i]);
          }
        }
        if (!(ok = mbar_wait_warp(&bars->s_full, sc & 1, ab))) break;
        tc_fence_after();
        {
          // P^T, 32 columns at a time, packed to bf16 pairs as they are produced
          uint32_t pk[32];
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            uint32_t sr[32];
            tmem_ld32(t_s + c2 * 32, sr);
            tmem_wait_ld();
            if (!warp_slow) {  // unmasked tile: p = 2^(s * scale * log2e + log2e * rel - lse2)
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float x0 = fmaf(__uint_as_float(sr[i]), a.scale_log2, nlr[c2 * 32 + i]);
                const float x1 = fmaf(__uint_as_float(sr[i + 1]), a.scale_log2, nlr[c2 * 32 + i + 1]);
                pk[c2 * 16 + i / 2] = pack_bf16x2(fast_exp2(x0), fast_exp2(x1));
              }
            } else {  // masked tile (any bias is already in nlr): p = 0 where masked
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const int c = c2 * 32 + i;
                const int cq = half * 64 + c;
                float p0 = fast_exp2(fmaf(__uint_as_float(sr[i]), a.scale_log2, nlr[c]));
                float p1 = fast_exp2(fmaf(__uint_as_float(sr[i + 1]), a.scale_log2, nlr[c + 1]));
                if (has_mask && (cq < c_lo || cq >= c_hi)) p0 = 0.f;
                if (has_mask && (cq + 1 < c_lo || cq + 1 >= c_hi)) p1 = 0.f;
                pk[c2 * 16 + i / 2] = pack_bf16x2(p0, p1);
              }
            }
          }
          __syncwarp();
          tmem_st32(t_s, pk);  // P^T over this half's first 32 columns (all 64 already read)
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full);
        // the next step's statistics, in flight while dS is computed
        const bool has_next = n + 1 < steps;
        float nv[4];
        if (has_next) {
          const int g1 = (n + 1) / blk.n_q;
          load_stats(kvh * group + g1, (blk.i_lo + n + 1 - g1 * blk.n_q) * kBM, nv);
        }
        float dlr[64];  // Delta of the 64 columns, loaded before the wait as -lse2 above
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          const float4 D = *reinterpret_cast<const float4*>(dl + c);
          dlr[c] = D.x;
          dlr[c + 1] = D.y;
          dlr[c + 2] = D.z;
          dlr[c + 3] = D.w;
        }
        if (!(ok = mbar_wait_warp(&bars->dp_full, sc & 1, ab))) break;
        tc_fence_after();
        // dS^T = P^T (dP^T - Delta) from the bf16 P^T in TMEM (the dV operand; the next S^T
        // overwrites it only after dK is issued), 32 columns at a time, in place over dP^T
        uint16_t* drel_h = a.drel + static_cast<long long>(h) * a.drel_sh;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t dr[32], pr[16];
          tmem_ld32(t_dp + c2 * 32, dr);
          tmem_ld16(t_s + c2 * 16, pr);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float* D = dlr + c2 * 32 + 2 * i;
            pk[i] = pack_bf16x2(__uint_as_float(pr[i] << 16) * (__uint_as_float(dr[2 * i]) - D[0]),
                                __uint_as_float(pr[i] & 0xffff0000u) * (__uint_as_float(dr[2 * i + 1]) - D[1]));
          }
          __syncwarp();
          tmem_st16(t_dp + c2 * 16, pk);  // columns [16 c2, 16 c2 + 16): already read
          if (warp_bias) {  // d rel: this key's band entries (dS of masked pairs is 0)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int cq = half * 64 + c2 * 32 + i;
              const int d = dq0 + cq;
              if (has_bias && d >= 0 && d < a.rel_extent && cq < sq - q0)
                drel_h[static_cast<long long>(q_start + q0 + cq) * a.drel_st + d] =
                    static_cast<uint16_t>((i & 1) ? (pk[i >> 1] >> 16) : (pk[i >> 1] & 0xffffu));
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->ds_full);
        if (has_next) store_stats((sc + 1) & 1, nv);  // that buffer's last reader was step n - 1
      }
      if (!ok) break;
      // epilogue: dV and scale * dK of this thread's key row, half of the columns
      if (!(ok = mbar_wait_warp(&bars->acc_full, ec & 1, ab))) break;
      ++ec;
      tc_fence_after();
      {
        uint32_t v0[32], v1[32];
        float f[64];
        tmem_ld32(tbase + lane_off + kColDV + half * 64, v0);
        tmem_ld32(tbase + lane_off + kColDV + half * 64 + 32, v1);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          f[c] = __uint_as_float(v0[c]);
          f[32 + c] = __uint_as_float(v1[c]);
        }
        if (key_valid) store_row64_bf16(dv_row, f, 1.f);
        tmem_ld32(tbase + lane_off + kColDK + half * 64, v0);
        tmem_ld32(tbase + lane_off + kColDK + half * 64 + 32, v1);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          f[c] = __uint_as_float(v0[c]);
          f[32 + c] = __uint_as_float(v1[c]);
        }
        if (key_valid) store_row64_bf16(dk_row, f, a.scale);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// --------------------------------------------------------------------------------------
// dQ
// --------------------------------------------------------------------------------------
namespace q {
constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemDO = kTile;
constexpr uint32_t kSmemK = 2 * kTile;  // 2 stages
constexpr uint32_t kSmemV = 4 * kTile;  // 2 stages
constexpr uint32_t kSmemBar = 6 * kTile;
// per elementwise warp, a 32-row x 32-column bf16 transpose buffer for the bias gather (rows
// 34 halfwords apart: conflict-free row writes and per-lane row reads)
constexpr uint32_t kBiasRowHalves = 34;
constexpr uint32_t kBiasWarpBytes = 32 * kBiasRowHalves * 2;
constexpr uint32_t kSmemBias = kSmemBar + 256;
constexpr uint32_t kSmemBytes = kSmemBias + 8 * kBiasWarpBytes;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr uint32_t kColS = 0, kColDP = 256, kColDQ = 384;  // S0 | S1 | dP | dQ

struct Bars {
  uint64_t qdo_full, qdo_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t dp_full, ds_full;
  uint64_t acc_full, acc_empty;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");
}  // namespace q

struct QTile {
  int j_lo, n_kv;
};

__device__ __forceinline__ QTile q_tile(const BackwardKernelArgs& a, int q0, int sq, int sk) {
  QTile t{0, 0};
  const int ms = a.align_bottom_right ? sk - sq : 0;
  const int r1 = min(q0 + kBM, sq);
  int hi = sk;
  if (a.causal) hi = min(hi, r1 + ms);
  int lo = 0;
  if (a.window_left >= 0) lo = max(0, q0 + ms - a.window_left);
  if (r1 > q0 && hi > lo) {
    t.j_lo = lo / kBN;
    t.n_kv = (hi + kBN - 1) / kBN - t.j_lo;
  }
  return t;
}

__global__ void __launch_bounds__(kThreads, 1)
    rel_attn_bwd_dq_kernel(const __grid_constant__ BackwardKernelArgs a,
                           const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v,
                           const __grid_constant__ CUtensorMap tm_do) {
  using namespace q;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kSmemBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid (query slots, heads, sequences) when the K / V stream over all kv heads outgrows L2,
  // otherwise (heads, sequences, query slots); as in the forward.
  const int h = a.slots_first_dq ? blockIdx.y : blockIdx.x;
  const int b = a.slots_first_dq ? blockIdx.z : blockIdx.y;
  const int slot0 = a.slots_first_dq ? blockIdx.x : blockIdx.z;
  const int slot_step = a.slots_first_dq ? gridDim.x : gridDim.z;
  const int kvh = h / (a.n_heads / a.kv_heads);
  const int q_start = a.cu_q[b];
  const int sq = a.cu_q[b + 1] - q_start;
  const int k_start = a.cu_k[b];
  const int sk = a.cu_k[b + 1] - k_start;
  const int n_qt = (sq + kBM - 1) / kBM;
  if (slot0 >= n_qt) return;

  if (threadIdx.x == 0) {
    mbar_init(&bars->qdo_full, 1);
    mbar_init(&bars->qdo_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
    }
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->ds_full, 8);
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 8);
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const AbortCtx ab{&bars->abort_flag, a.status, kStatusBackwardTimeout};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t qc = 0, kc = 0, vc = 0;
      const uint64_t pol_kv = l2_policy_evict_last();
      const uint64_t pol_q = l2_policy_evict_first();
      bool ok = true;
      for (int slot = slot0; slot < n_qt && ok; slot += slot_step) {
        const int q0 = (n_qt - 1 - slot) * kBM;
        const QTile t = q_tile(a, q0, sq, sk);
        if (t.n_kv == 0) continue;
        if (!(ok = mbar_wait(&bars->qdo_empty, (qc & 1) ^ 1, ab))) break;
        mbar_arrive_expect_tx(&bars->qdo_full, 2 * kTile);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_3d_hint(smem + kSmemQ + hf * kHalf, &tm_q, &bars->qdo_full, hf * 64, h,
                           q_start + q0, pol_q);
          tma_load_3d_hint(smem + kSmemDO + hf * kHalf, &tm_do, &bars->qdo_full, hf * 64, h,
                           q_start + q0, pol_q);
        }
        ++qc;
        for (int j = 0; j < t.n_kv && ok; ++j) {
          const int row = k_start + (t.j_lo + j) * kBN;
          const uint32_t ks = kc & 1;
          if (!(ok = mbar_wait(&bars->k_empty[ks], ((kc >> 1) & 1) ^ 1, ab))) break;
          mbar_arrive_expect_tx(&bars->k_full[ks], kTile);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d_hint(smem + kSmemK + ks * kTile + hf * kHalf, &tm_k, &bars->k_full[ks],
                             hf * 64, kvh, row, pol_kv);
          ++kc;
          const uint32_t vs = vc & 1;
          if (!(ok = mbar_wait(&bars->v_empty[vs], ((vc >> 1) & 1) ^ 1, ab))) break;
          mbar_arrive_expect_tx(&bars->v_full[vs], kTile);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d_hint(smem + kSmemV + vs * kTile + hf * kHalf, &tm_v, &bars->v_full[vs],
                             hf * 64, kvh, row, pol_kv);
          ++vc;
        }
      }
      if (qc > 0) mbar_wait(&bars->qdo_full, (qc - 1) & 1, ab);
      for (uint32_t i = 0; i < 2 && i < kc; ++i) {
        const uint32_t last = kc - 1 - i;
        mbar_wait(&bars->k_full[last & 1], (last >> 1) & 1, ab);
      }
      for (uint32_t i = 0; i < 2 && i < vc; ++i) {
        const uint32_t last = vc - 1 - i;
        mbar_wait(&bars->v_full[last & 1], (last >> 1) & 1, ab);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      uint32_t qc = 0, kc = 0, vc = 0, sc = 0, ec = 0;
      const uint32_t q_addr = smem_u32(smem + kSmemQ);
      const uint32_t do_addr = smem_u32(smem + kSmemDO);
      const uint32_t k_addr = smem_u32(smem + kSmemK);
      const uint32_t v_addr = smem_u32(smem + kSmemV);
      bool ok = true;
      for (int slot = slot0; slot < n_qt && ok; slot += slot_step) {
        const int q0 = (n_qt - 1 - slot) * kBM;
        const QTile t = q_tile(a, q0, sq, sk);
        if (t.n_kv == 0) continue;
        if (!(ok = mbar_wait(&bars->qdo_full, qc & 1, ab))) break;
        ++qc;
        // first tile: S_0 = Q K_0^T, dP_0 = dO V_0^T
        if (!(ok = mbar_wait(&bars->k_full[kc & 1], (kc >> 1) & 1, ab))) break;
        tc_fence_after();
        mma_kk(tbase + kColS + (sc & 1) * 128, q_addr, k_addr + (kc & 1) * kTile);
        umma_commit(&bars->s_full[sc & 1]);
        if (!(ok = mbar_wait(&bars->v_full[vc & 1], (vc >> 1) & 1, ab))) break;
        tc_fence_after();
        mma_kk(tbase + kColDP, do_addr, v_addr + (vc & 1) * kTile);
        umma_commit(&bars->dp_full);
        for (int j = 0; j < t.n_kv && ok; ++j) {
          const uint32_t ks = kc & 1, vs = vc & 1;
          if (j + 1 < t.n_kv) {  // next tile's S into the other buffer, overlapping this dS
            const uint32_t kn = kc + 1;
            if (!(ok = mbar_wait(&bars->k_full[kn & 1], (kn >> 1) & 1, ab))) break;
            tc_fence_after();
            mma_kk(tbase + kColS + ((sc + 1) & 1) * 128, q_addr, k_addr + (kn & 1) * kTile);
            umma_commit(&bars->s_full[(sc + 1) & 1]);
          }
          if (j == 0 && !(ok = mbar_wait(&bars->acc_empty, (ec & 1) ^ 1, ab))) break;
          if (!(ok = mbar_wait(&bars->ds_full, sc & 1, ab))) break;
          tc_fence_after();
          mma_tk(tbase + kColDQ, tbase + kColS + (sc & 1) * 128, k_addr + ks * kTile, j > 0);
          umma_commit(&bars->k_empty[ks]);
          umma_commit(&bars->v_empty[vs]);
          ++kc;
          ++vc;
          ++sc;
          if (j + 1 < t.n_kv) {
            if (!(ok = mbar_wait(&bars->v_full[vc & 1], (vc >> 1) & 1, ab))) break;
            tc_fence_after();
            mma_kk(tbase + kColDP, do_addr, v_addr + (vc & 1) * kTile);
            umma_commit(&bars->dp_full);
          }
        }
        if (!ok) break;
        umma_commit(&bars->acc_full);
        umma_commit(&bars->qdo_empty);
        ++ec;
      }
      umma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, ab);
    }
  } else {
    // ------------------------------------------------------------------ elementwise + epilogue
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int ms = a.align_bottom_right ? sk - sq : 0;
    const int bs = a.align_bottom_right ? sk - sq : sq - sk;
    uint16_t* bias_buf = reinterpret_cast<uint16_t*>(smem + kSmemBias + (warp - 2) * kBiasWarpBytes);
    uint32_t sc = 0, ec = 0;
    bool ok = true;
    for (int slot = slot0; slot < n_qt && ok; slot += slot_step) {
      const int q0 = (n_qt - 1 - slot) * kBM;
      const QTile t = q_tile(a, q0, sq, sk);
      const int qi = q0 + r;
      const bool row_valid = qi < sq;
      IFA4_DBG_CHECK(a.status, !row_valid || q_start + qi < a.total_q);  // report only
      uint16_t* dq_row = a.dq + static_cast<long long>(q_start + qi) * a.dq_st +
                         static_cast<long long>(h) * a.dq_sh + half * 64;
      if (t.n_kv == 0) {
        if (row_valid) store_zero_row64(dq_row);
        continue;
      }
      float lse2 = 0.f, dlt = 0.f;
      if (row_valid) {
        const long long tok = q_start + qi;
        lse2 = a.lse[static_cast<long long>(h) * a.lse_sh + tok * a.lse_st] * kLog2e;
        dlt = a.delta[static_cast<long long>(h) * a.total_q + tok];
      }
      const uint16_t* rel_row = a.rel + static_cast<long long>(q_start + qi) * a.rel_st +
                                static_cast<long long>(h) * a.rel_sh;
      int key_hi = sk;
      if (a.causal) key_hi = min(key_hi, qi + ms + 1);
      int key_lo = a.window_left >= 0 ? max(0, qi + ms - a.window_left) : 0;
      if (!row_valid) key_hi = key_lo = 0;
      const int dmax = qi + bs;  // bias distance at key 0
      for (int j = 0; j < t.n_kv; ++j, ++sc) {
        const int k0 = (t.j_lo + j) * kBN;
        const uint32_t t_s = tbase + lane_off + kColS + (sc & 1) * 128 + half * 64;
        const int cb = half * 64;                       // first column of this half
        const int cl = key_lo - k0, ch = key_hi - k0;   // visible columns [cl, ch)
        const bool has_mask = cl > cb || ch < cb + 64;
        const int bl = dmax - a.rel_extent + 1 - k0;    // first column with bias
        const int bh = dmax - k0;                       // last column with bias
        const bool has_bias = row_valid && bl <= cb + 63 && bh >= cb;
        // vector bias path: this row's windows for both chunks, loaded while S is computed
        uint32_t bwin[2][20];
        if (a.bias_vec && __any_sync(0xffffffffu, has_bias)) {
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            const int c0 = cb + c2 * 32;
            load_bias_window(rel_row, bh, c0 >> 5, a.rel_extent,
                             has_bias && c0 + 31 >= bl && c0 <= bh, bwin[c2]);
          }
        }
        if (!(ok = mbar_wait_warp(&bars->s_full[sc & 1], (sc >> 1) & 1, ab))) break;
        tc_fence_after();
        float p[64];
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t sr[32];
          tmem_ld32(t_s + c2 * 32, sr);
          tmem_wait_ld();
          float x[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(sr[i]) * a.scale_log2 - lse2;
          const int c0 = cb + c2 * 32;  // absolute first column of this chunk
          const bool chunk_bias = has_bias && c0 + 31 >= bl && c0 <= bh;
          if (a.bias_vec) {
            if (__any_sync(0xffffffffu, chunk_bias)) add_bias_window(bwin[c2], bh, c0 >> 5, x);
          } else if (__any_sync(0xffffffffu, chunk_bias)) {
            // the warp gathers its 32 rows' bias for these 32 columns (coalesced row reads),
            // transposes through shared memory, and each lane adds its own row
            uint16_t v[32];
#pragma unroll
            for (int tr = 0; tr < 32; ++tr) {
              const int qi_t = qi - lane + tr;
              const int d = qi_t + bs - k0 - (c0 + lane);
              v[tr] = 0;
              if (qi_t < sq && d >= 0 && d < a.rel_extent)
                v[tr] = __ldg(rel_row + static_cast<long long>(tr - lane) * a.rel_st + d);
            }
#pragma unroll
            for (int tr = 0; tr < 32; ++tr) bias_buf[tr * kBiasRowHalves + lane] = v[tr];
            __syncwarp();
            const uint32_t* w = reinterpret_cast<const uint32_t*>(bias_buf) + lane * (kBiasRowHalves / 2);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const uint32_t pr = w[k];
              x[2 * k] += __uint_as_float(pr << 16) * kLog2e;
              x[2 * k + 1] += __uint_as_float(pr & 0xffff0000u) * kLog2e;
            }
            __syncwarp();
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) p[c2 * 32 + i] = fast_exp2(x[i]);
          if (has_mask) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = c0 + i;
              if (col < cl || col >= ch) p[c2 * 32 + i] = 0.f;
            }
          }
        }
        if (!(ok = mbar_wait_warp(&bars->dp_full, sc & 1, ab))) break;
        tc_fence_after();
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {  // dS over this half's first 32 columns of the S buffer
          uint32_t dr[32];
          tmem_ld32(tbase + lane_off + kColDP + half * 64 + c2 * 32, dr);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack_bf16x2(p[c2 * 32 + 2 * i] * (__uint_as_float(dr[2 * i]) - dlt),
                                p[c2 * 32 + 2 * i + 1] * (__uint_as_float(dr[2 * i + 1]) - dlt));
          __syncwarp();
          tmem_st16(t_s + c2 * 16, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->ds_full);
      }
      if (!ok) break;
      if (!(ok = mbar_wait_warp(&bars->acc_full, ec & 1, ab))) break;
      ++ec;
      tc_fence_after();
      {
        uint32_t v0[32], v1[32];
        float f[64];
        tmem_ld32(tbase + lane_off + kColDQ + half * 64, v0);
        tmem_ld32(tbase + lane_off + kColDQ + half * 64 + 32, v1);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          f[c] = __uint_as_float(v0[c]);
          f[32 + c] = __uint_as_float(v1[c]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acc_empty);
        if (row_valid) store_row64_bf16(dq_row, f, a.scale);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace bwd

cudaError_t launch_backward_sm100(const BackwardKernelArgs& args, const CUtensorMap& tm_q,
                                  const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                  const CUtensorMap& tm_do, int q_slots, int k_slots,
                                  cudaStream_t stream) {
  static std::atomic<bool> kv_attr[64], q_attr[64];
  cudaError_t e = set_smem_limit_once(bwd::rel_attn_bwd_dkdv_kernel, bwd::kv::kSmemAlloc, kv_attr);
  if (e != cudaSuccess) return e;
  e = set_smem_limit_once(bwd::rel_attn_bwd_dq_kernel, bwd::q::kSmemAlloc, q_attr);
  if (e != cudaSuccess) return e;
  const long long rows = args.total_q * args.n_heads;
  if (rows > 0) {
    const long long blocks = (rows + 7) / 8;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    bwd::rel_attn_bwd_prep_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(args);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const dim3 kgrid = args.slots_first_dkdv ? dim3(k_slots, args.kv_heads, args.batch)
                                           : dim3(args.kv_heads, args.batch, k_slots);
  bwd::rel_attn_bwd_dkdv_kernel<<<kgrid, bwd::kThreads, bwd::kv::kSmemAlloc, stream>>>(
      args, tm_q, tm_k, tm_v, tm_do);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 qgrid = args.slots_first_dq ? dim3(q_slots, args.n_heads, args.batch)
                                         : dim3(args.n_heads, args.batch, q_slots);
  bwd::rel_attn_bwd_dq_kernel<<<qgrid, bwd::kThreads, bwd::q::kSmemAlloc, stream>>>(
      args, tm_q, tm_k, tm_v, tm_do);
  return cudaGetLastError();
}

}  // namespace ifa4
