// Split-KV single-token decode for sm_100a: an HBM-streaming kernel plus a combine kernel.
//
// Grid (num_splits, kv_heads * head_blocks, batch); one CTA streams a chunk set of one
// sequence's visible keys for up to 16 query heads of ONE GQA group, so every K/V byte is read
// from HBM once per group rather than once per query head (the reference decode kernel,
// triton_kernel_decode.py:66-118, re-reads K/V for every head).
//   warp 4      TMA producer: 64-key K and V tiles (128-byte swizzle, 128-bit granules, no
//               multicast) into a 3-stage shared-memory ring.
//   warps 0-3   consumers: each takes 16 keys of every tile.  S = Q K^T and O += P V run on
//               warp-level bf16 MMAs (m16n8k16, fp32 accumulate) with the query heads in the M
//               dimension; row max / sum use quad shuffles; online softmax in the exp2 domain
//               with the fused relative-bias gather.
// The four warps' (max, sum, O) states are merged in shared memory; with one split the CTA
// writes the bf16 output, otherwise a normalised fp32 partial and its log2-sum-exp, which
// rel_attn_decode_combine_kernel merges.
//
// Paged KV cache (kPaged): the whole producer warp runs, fetching the next tile's page numbers
// from the block table while the current tile is issued; a 64-key tile is loaded as 64 / box
// units of box = min(page_size, 64) rows (one 4-D TMA box per unit, tensor and 64-dim half),
// units past the sequence's end load zeros, and tiles start at the window's first key rounded
// down to the box size.  V values of keys past the sequence's end (unused cache slots, possibly
// NaN) are zeroed in the B fragments before the P.V product.
//
// Decode is bandwidth-bound (about 4 FLOP per K/V byte for a group of 4), so the roofline is
// HBM; the warp-level MMA keeps the issue cost per key small.  Semantics follow the oracle
// (reference.py:27-39) for sq = 1.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "ifa4_internal.h"
#include "ifa4_ptx.cuh"

namespace ifa4 {
namespace decode {

constexpr int kTileKeys = 64;
constexpr int kStages = 3;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr uint32_t kHalf = kTileKeys * 128;             // 64 rows x 128 B
constexpr uint32_t kKVTile = 2 * kHalf;                 // 64 keys x 256 B
constexpr uint32_t kStageBytes = 2 * kKVTile;           // K + V
constexpr uint32_t kSmemBar = kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kSmemBar + 128;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr float kLog2e = 1.4426950408889634f;

struct Bars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int abort_flag;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Address of the 16-byte granule (row, chunk) of a 64-row tile stored as two 128-B-swizzled
// halves of 64 dims (chunk 0..15 over the 128 dims).
__device__ __forceinline__ uint32_t sw128_addr(uint32_t base, int row, int chunk) {
  return base + (chunk >> 3) * kHalf + row * 128 + ((((chunk & 7) ^ (row & 7))) << 4);
}

struct SeqInfo {
  int q_row, k_start, sk, lo, hi, base, nchunks;  // chunks start at base + c * chunk_len
};

template <bool kPaged>
__device__ __forceinline__ SeqInfo seq_info(const DecodeKernelArgs& a, int b) {
  SeqInfo s;
  s.q_row = a.cu_q[b];
  s.k_start = a.cu_k[b];
  s.sk = a.cu_k[b + 1] - s.k_start;
  const int ms = a.align_bottom_right ? s.sk - 1 : 0;  // sq = 1, q_pos = 0
  s.hi = s.sk;
  if (a.causal) s.hi = min(s.hi, ms + 1);
  s.lo = a.window_left >= 0 ? max(0, ms - a.window_left) : 0;
  s.base = kPaged ? s.lo & ~((1 << a.box_shift) - 1) : s.lo;
  s.nchunks = s.hi > s.lo ? (s.hi - s.base + a.chunk_len - 1) / a.chunk_len : 0;
  return s;
}

template <bool kPaged>
__global__ void __launch_bounds__(kThreads, 2)
    rel_attn_decode_kernel(const __grid_constant__ DecodeKernelArgs a,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kSmemBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int head_blocks = (a.group + a.heads_per_cta - 1) / a.heads_per_cta;
  const int kvh = blockIdx.y / head_blocks;
  const int hblk = blockIdx.y % head_blocks;
  const int h0 = kvh * a.group + hblk * a.heads_per_cta;
  const int nh = min(a.heads_per_cta, a.group - hblk * a.heads_per_cta);
  const int b = blockIdx.z;
  const SeqInfo si = seq_info<kPaged>(a, b);
  const int bs = a.align_bottom_right ? si.sk - 1 : 1 - si.sk;  // bias distance at key 0

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], kConsumerWarps);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const AbortCtx ab{&bars->abort_flag, a.status, kStatusDecodeTimeout};

  // per-thread softmax state (consumer warps): rows g = lane/4 and g + 8
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  if (kPaged && warp == kConsumerWarps) {
    // ---------------------------------------------------------------- paged TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    const uint64_t pol = l2_policy_evict_first();
    const int box = 1 << a.box_shift;
    const int units = kTileKeys >> a.box_shift;
    const int page_mask = (1 << a.page_shift) - 1;
    const int32_t* bt = a.block_table + static_cast<long long>(b) * a.bt_stride;
    // page of unit `lane` of the tile at key t0; -1 past the end or for an invalid entry
    auto unit_block = [&](int t0) {
      const int key = t0 + lane * box;
      int blk = -1;
      if (lane < units && key < si.sk) {
        blk = __ldg(bt + (key >> a.page_shift));
        if (blk < 0 || blk >= a.num_pages) blk = -1;
      }
      return blk;
    };
    uint32_t n = 0;
    int c = split;
    int t0 = si.base + c * a.chunk_len;
    int blk = c < si.nchunks ? unit_block(t0) : -1;
    while (c < si.nchunks) {
      const int c1 = min(si.hi, si.base + c * a.chunk_len + a.chunk_len);
      int nc = c, nt0 = t0 + kTileKeys;  // the tile after this one, in consumer order
      if (nt0 >= c1) {
        nc = c + gridDim.x;
        nt0 = si.base + nc * a.chunk_len;
      }
      const int nblk = nc < si.nchunks ? unit_block(nt0) : -1;  // in flight across the wait
      const uint32_t st = n % kStages;
      if (!mbar_wait_warp(&bars->empty[st], ((n / kStages) & 1) ^ 1, ab)) break;
      if (lane == 0) mbar_arrive_expect_tx(&bars->full[st], kStageBytes);
      __syncwarp();
      if (lane < units) {
        uint8_t* base = smem + st * kStageBytes + lane * box * 128;
        const int in_page = (t0 + lane * box) & page_mask;
        const int page = blk >= 0 ? blk : a.num_pages;  // out of range: TMA writes zeros
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_4d_hint(base + hf * kHalf, &tm_k, &bars->full[st], hf * 64, kvh, in_page,
                           page, pol);
          tma_load_4d_hint(base + kKVTile + hf * kHalf, &tm_v, &bars->full[st], hf * 64, kvh,
                           in_page, page, pol);
        }
      }
      ++n;
      c = nc;
      t0 = nt0;
      blk = nblk;
    }
    if (lane == 0) {  // drain the last use of every stage
      for (uint32_t i = 0; i < kStages && i < n; ++i) {
        const uint32_t last = n - 1 - i;
        mbar_wait(&bars->full[last % kStages], (last / kStages) & 1, ab);
      }
    }
  } else if (warp == kConsumerWarps) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint64_t pol = l2_policy_evict_first();
      uint32_t n = 0;
      bool ok = true;
      for (int c = split; c < si.nchunks && ok; c += gridDim.x) {
        const int c0 = si.base + c * a.chunk_len;
        const int c1 = min(si.hi, c0 + a.chunk_len);
        for (int t0 = c0; t0 < c1; t0 += kTileKeys, ++n) {
          const uint32_t st = n % kStages;
          const uint32_t ph = (n / kStages) & 1;
          if (!(ok = mbar_wait(&bars->empty[st], ph ^ 1, ab))) break;
          mbar_arrive_expect_tx(&bars->full[st], kStageBytes);
          uint8_t* base = smem + st * kStageBytes;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            tma_load_3d_hint(base + hf * kHalf, &tm_k, &bars->full[st], hf * 64, kvh,
                             si.k_start + t0, pol);
            tma_load_3d_hint(base + kKVTile + hf * kHalf, &tm_v, &bars->full[st], hf * 64, kvh,
                             si.k_start + t0, pol);
          }
        }
      }
      // drain the last use of every stage
      for (uint32_t i = 0; i < kStages && i < n; ++i) {
        const uint32_t last = n - 1 - i;
        mbar_wait(&bars->full[last % kStages], (last / kStages) & 1, ab);
      }
    }
  } else {
    // ---------------------------------------------------------------- consumers
    const int g = lane >> 2;
    const int qd = lane & 3;
    // Q A-fragments: rows = heads h0 + g (+8), k = dims.
    uint32_t qa[8][4];
    const uint32_t* qrow0 = reinterpret_cast<const uint32_t*>(
        a.q + static_cast<long long>(si.q_row) * a.q_st + static_cast<long long>(h0 + g) * a.q_sh);
    const uint32_t* qrow1 = reinterpret_cast<const uint32_t*>(
        a.q + static_cast<long long>(si.q_row) * a.q_st +
        static_cast<long long>(h0 + g + 8) * a.q_sh);
    const bool r0v = g < nh, r1v = g + 8 < nh;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qa[kk][0] = r0v ? __ldg(qrow0 + kk * 8 + qd) : 0u;
      qa[kk][1] = r1v ? __ldg(qrow1 + kk * 8 + qd) : 0u;
      qa[kk][2] = r0v ? __ldg(qrow0 + kk * 8 + 4 + qd) : 0u;
      qa[kk][3] = r1v ? __ldg(qrow1 + kk * 8 + 4 + qd) : 0u;
    }
    const uint16_t* relr[2];
    relr[0] = a.rel + static_cast<long long>(si.q_row) * a.rel_st +
              static_cast<long long>(h0 + g) * a.rel_sh;
    relr[1] = a.rel + static_cast<long long>(si.q_row) * a.rel_st +
              static_cast<long long>(h0 + g + 8) * a.rel_sh;
    uint32_t n = 0;
    bool ok = true;
    for (int c = split; c < si.nchunks && ok; c += gridDim.x) {
      const int c0 = si.base + c * a.chunk_len;
      const int c1 = min(si.hi, c0 + a.chunk_len);
      for (int t0 = c0; t0 < c1; t0 += kTileKeys, ++n) {
        const uint32_t st = n % kStages;
        if (!(ok = mbar_wait_warp(&bars->full[st], (n / kStages) & 1, ab))) break;
        const uint32_t kbase = smem_u32(smem + st * kStageBytes);
        const uint32_t vbase = kbase + kKVTile;
        const int wrow = warp * 16;  // this warp's 16 keys within the tile
        // ---- S = Q K^T for 16 keys (two n8 tiles)
        float s[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
        {
          const int mi = lane >> 3;  // which 8x8 matrix this lane addresses
          const int krow = wrow + (mi >> 1) * 8 + (lane & 7);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(sw128_addr(kbase, krow, 2 * kk + (mi & 1)), b0, b1, b2, b3);
            mma_bf16(s[0], qa[kk], b0, b1);
            mma_bf16(s[1], qa[kk], b2, b3);
          }
        }
        // ---- scale, bias, mask
        const int kt = t0 + wrow;  // local key index of column 0 of this warp's slice
        float x[2][2][2];          // [row r][ntile][e]
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            x[0][nt][e] = s[nt][e] * a.scale_log2;
            x[1][nt][e] = s[nt][2 + e] * a.scale_log2;
          }
        if (bs - (kt + 15) < a.rel_extent && bs - kt >= 0) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            if (!(r == 0 ? r0v : r1v)) continue;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int d = bs - (kt + nt * 8 + 2 * qd + e);
                if (d >= 0 && d < a.rel_extent)
                  x[r][nt][e] += bf16_bits_to_float(__ldg(relr[r] + d)) * kLog2e;
              }
          }
        }
        if (kt < si.lo || kt + 16 > si.hi) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int key = kt + nt * 8 + 2 * qd + e;
              if (key < si.lo || key >= si.hi) x[0][nt][e] = x[1][nt][e] = -INFINITY;
            }
        }
        // ---- online softmax per row
        uint32_t pa[4];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          float mt = fmaxf(fmaxf(x[r][0][0], x[r][0][1]), fmaxf(x[r][1][0], x[r][1][1]));
          mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
          mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
          const float m_new = fmaxf(m_r[r], mt);
          // m_r = -inf, m_new finite -> alpha = 0; both -inf -> nothing seen yet, alpha = 1
          const float alpha = m_new == -INFINITY ? 1.f : fast_exp2(m_r[r] - m_new);
          const float m_use = m_new == -INFINITY ? 0.f : m_new;
          m_r[r] = m_new;
          const float p00 = fast_exp2(x[r][0][0] - m_use), p01 = fast_exp2(x[r][0][1] - m_use);
          const float p10 = fast_exp2(x[r][1][0] - m_use), p11 = fast_exp2(x[r][1][1] - m_use);
          l_r[r] = l_r[r] * alpha + (p00 + p01 + p10 + p11);
#pragma unroll
          for (int dt = 0; dt < 16; ++dt) {
            o[dt][2 * r] *= alpha;
            o[dt][2 * r + 1] *= alpha;
          }
          pa[r] = pack_bf16x2(p00, p01);      // a0 (r=0) / a1 (r=1): keys 0..7 of the k16
          pa[2 + r] = pack_bf16x2(p10, p11);  // a2 / a3: keys 8..15
        }
        // ---- O += P V  (V^T fragments via transposed ldmatrix).  The bias/mask code above
        // branches per lane; ldmatrix/mma are .sync.aligned: reconverge the warp first.
        // Paged cache: keys past the sequence's end may sit in unused (even NaN) cache slots;
        // this lane's B fragments hold keys kt + 2qd (+1) (b0, b2; low, high half) and
        // kt + 8 + 2qd (+1) (b1, b3).
        uint32_t vm0 = 0xffffffffu, vm1 = 0xffffffffu;
        if (kPaged && kt + 16 > si.sk) {
          const int k0 = kt + 2 * qd;
          vm0 = (k0 < si.sk ? 0x0000ffffu : 0u) | (k0 + 1 < si.sk ? 0xffff0000u : 0u);
          vm1 = (k0 + 8 < si.sk ? 0x0000ffffu : 0u) | (k0 + 9 < si.sk ? 0xffff0000u : 0u);
        }
        __syncwarp();
        {
          const int mi = lane >> 3;
          const int vrow = wrow + (mi & 1) * 8 + (lane & 7);
#pragma unroll
          for (int dt = 0; dt < 16; dt += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(sw128_addr(vbase, vrow, dt + (mi >> 1)), b0, b1, b2, b3);
            if (kPaged) {
              b0 &= vm0;
              b1 &= vm1;
              b2 &= vm0;
              b3 &= vm1;
            }
            mma_bf16(o[dt], pa, b0, b1);
            mma_bf16(o[dt + 1], pa, b2, b3);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->empty[st]);
      }
    }
    // full row sums across the quad
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
      l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
    }
  }

  // ------------------------------------------------------------------ merge the 4 warps
  __syncthreads();  // all TMA traffic drained (producer) and all stages consumed
  float* mo = reinterpret_cast<float*>(smem);                       // [4][16][128]
  float* mm = mo + kConsumerWarps * 16 * 128;                       // [4][16]
  float* ml = mm + kConsumerWarps * 16;                             // [4][16]
  if (warp < kConsumerWarps) {
    const int g = lane >> 2, qd = lane & 3;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      if (qd == 0) {
        mm[warp * 16 + row] = m_r[r];
        ml[warp * 16 + row] = l_r[r];
      }
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        mo[(warp * 16 + row) * 128 + dt * 8 + 2 * qd] = o[dt][2 * r];
        mo[(warp * 16 + row) * 128 + dt * 8 + 2 * qd + 1] = o[dt][2 * r + 1];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const int d = threadIdx.x;
    for (int row = 0; row < nh; ++row) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mm[w * 16 + row]);
      float L = 0.f, acc = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float f = fast_exp2(mm[w * 16 + row] - M);
          L += ml[w * 16 + row] * f;
          acc += mo[(w * 16 + row) * 128 + d] * f;
        }
      }
      const int h = h0 + row;
      const float val = L > 0.f ? acc / L : 0.f;
      if (!IFA4_DBG_CHECK(a.status, si.q_row >= 0 && si.q_row < a.batch && h < a.n_heads)) {
        // a bad query row or head: nothing is stored
      } else if (gridDim.x == 1) {
        uint16_t* dst = a.out + static_cast<long long>(si.q_row) * a.out_st +
                        static_cast<long long>(h) * a.out_sh + d;
        __nv_bfloat16 bv = __float2bfloat16_rn(val);
        *dst = *reinterpret_cast<uint16_t*>(&bv);
        if (d == 0 && a.lse != nullptr)
          a.lse[static_cast<long long>(h) * a.lse_sh + static_cast<long long>(si.q_row) * a.lse_st] =
              L > 0.f ? (M + __log2f(L)) * 0.6931471805599453f : -INFINITY;
      } else {
        const long long idx = (static_cast<long long>(b) * a.n_heads + h) * gridDim.x + split;
        a.ws_o[idx * 128 + d] = val;
        if (d == 0) a.ws_lse[idx] = L > 0.f ? M + __log2f(L) : -INFINITY;
      }
    }
  }
}

// Merge num_splits normalised partials per (sequence, head): weights 2^(lse_s - max lse).
__global__ void __launch_bounds__(128)
    rel_attn_decode_combine_kernel(const __grid_constant__ DecodeKernelArgs a) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int S = a.num_splits;
  const long long base = (static_cast<long long>(b) * a.n_heads + h) * S;
  if (!IFA4_DBG_CHECK(a.status, a.cu_q[b] >= 0 && a.cu_q[b] < a.batch)) return;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, a.ws_lse[base + s]);
  float wsum = 0.f, acc = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < S; ++s) {
      const float w = fast_exp2(a.ws_lse[base + s] - M);
      wsum += w;
      acc += w * a.ws_o[(base + s) * 128 + d];
    }
  }
  const float val = wsum > 0.f ? acc / wsum : 0.f;
  const int q_row = a.cu_q[b];
  if (d == 0 && a.lse != nullptr)  // log2-sum-exp of the partials -> natural log
    a.lse[static_cast<long long>(h) * a.lse_sh + static_cast<long long>(q_row) * a.lse_st] =
        wsum > 0.f ? (M + __log2f(wsum)) * 0.6931471805599453f : -INFINITY;
  __nv_bfloat16 bv = __float2bfloat16_rn(val);
  a.out[static_cast<long long>(q_row) * a.out_st + static_cast<long long>(h) * a.out_sh + d] =
      *reinterpret_cast<uint16_t*>(&bv);
}

}  // namespace decode

cudaError_t launch_decode_sm100(const DecodeKernelArgs& args, const CUtensorMap& tm_k,
                                const CUtensorMap& tm_v, cudaStream_t stream) {
  static std::atomic<bool> attr_contig[64], attr_paged[64];
  cudaError_t se = set_smem_limit_once(decode::rel_attn_decode_kernel<false>, decode::kSmemAlloc,
                                       attr_contig);
  if (se == cudaSuccess)
    se = set_smem_limit_once(decode::rel_attn_decode_kernel<true>, decode::kSmemAlloc, attr_paged);
  if (se != cudaSuccess) return se;
  const int head_blocks = (args.group + args.heads_per_cta - 1) / args.heads_per_cta;
  dim3 grid(args.num_splits, args.kv_heads * head_blocks, args.batch);
  if (args.block_table != nullptr)
    decode::rel_attn_decode_kernel<true><<<grid, decode::kThreads, decode::kSmemAlloc, stream>>>(
        args, tm_k, tm_v);
  else
    decode::rel_attn_decode_kernel<false><<<grid, decode::kThreads, decode::kSmemAlloc, stream>>>(
        args, tm_k, tm_v);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || args.num_splits == 1) return e;
  dim3 cgrid(args.n_heads, args.batch);
  decode::rel_attn_decode_combine_kernel<<<cgrid, 128, 0, stream>>>(args);
  return cudaGetLastError();
}

}  // namespace ifa4
