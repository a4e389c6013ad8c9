// rel_logits producer for sm_100a: the step in front of the attention in the Inkling layer
// (RelLogitsProj and the log-tau scaling; the reference repository holds only a diagram of it,
// outputs/architecture.md:51-64), fused into one HBM-bound kernel:
//   rel[t, h, e] = bf16( tau(pos_t) * sum_{j < 16} r[t, h, j] * W_h[j, e] )
//   tau(p)       = 1 + alpha * log(max((p + 1) / nf, 1))
//
// Work: quads of 128 tokens x 4 consecutive heads x 128 rel columns (one column block), ordered
// token tile first, so the CTAs running at one time write whole token rows of rel.  The quad's r
// rows form one K-major 128-byte-swizzled tile (row i = token i; head k's 16 features at bytes
// 32k..32k+31), loaded with one coalesced 128-byte row per thread, so the four heads' A operands
// are the same tile at four 32-byte K offsets.  Per head (unit): the 16 x 128 slice of W_h is
// the MN-major B operand in W's own layout (two 64-column halves of 16 swizzled 128-byte rows);
// one tcgen05.mma (M = N = 128, K = 16, fp32 accumulation) writes the 128 x 128 products to TMEM;
// each thread drains its TMEM lane (one token), multiplies by tau (packed f32x2), rounds to bf16
// and writes a swizzled staging tile that two TMA stores of 64 columns write to rel.  Four CTAs
// per SM (52 KB shared memory and 128 TMEM columns each) overlap one another's MMA, drain and
// stores; each thread fetches the next quad's r row and the next unit's weight chunk into
// registers while the current unit runs.  Quads advance by a precomputed step (no 64-bit
// division in the loop).
//
// Measured alternatives (32k tokens x 32 heads x R = 128, steady state): one unit (one head) per
// CTA iteration with a 32-byte r load per token and unit: 66 us (the scattered 32-byte r reads
// alone took 32 us); a persistent warp-specialised kernel (one CTA per SM, cp.async loader warp,
// MMA warp, 8 epilogue warps, four TMEM accumulators, four TMA stores in flight per half) 74 us,
// and 80 us with plain coalesced stores in place of TMA stores.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ifa4_internal.h"
#include "ifa4_ptx.cuh"

namespace ifa4 {
namespace rl {

constexpr int kRows = 128;      // tokens per quad (UMMA M; one TMEM lane per token)
constexpr int kCols = 128;      // rel columns per unit (UMMA N)
constexpr int kThreads = 128;
constexpr int kCtasPerSm = 4;
constexpr uint32_t kTile = 128u * 128u;  // 128 rows x 128 B
constexpr uint32_t kBHalf = 16u * 128u;  // 16 K rows x 128 B (64 rel columns)
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kIdesc = idesc_bf16_f32(128, 128, /*b_mn_major=*/true);
static_assert(kCtasPerSm == kRelLogitsCtasPerSm, "grid sizing in the C ABI layer");
static_assert(kCtasPerSm * kTmemCols <= 512, "TMEM columns per SM");

struct Smem {
  uint8_t a[kTile];       // row i: token i, head k's 16 features at bytes 32k.., SW128 (K-major)
  uint8_t b[2][kBHalf];   // W_h rows j = 0..15, 64 columns per half, SW128 (MN-major)
  uint8_t out[2][kTile];  // bf16 result: columns [0, 64) and [64, 128), SW128 TMA boxes
  uint64_t mma_bar;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr uint32_t kSmemAlloc = sizeof(Smem) + 1024;  // + slack for 1024-byte alignment

__device__ __forceinline__ void st_shared_v4(uint8_t* p, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(uint64_t pair) {
  float lo, hi;
  f2_unpack(pair, lo, hi);
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Position of token t in its sequence (see IFA4RelLogitsParams) and its tau.
__device__ __forceinline__ float row_tau(const RelLogitsKernelArgs& a, long long t) {
  if (a.alpha == 0.f || t >= a.total_q) return 1.f;
  long long pos = t;
  if (a.cu_q != nullptr) {
    int lo = 0, hi = a.batch - 1;  // largest b with cu_q[b] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(a.cu_q + mid) <= t) lo = mid; else hi = mid - 1;
    }
    const int q0 = __ldg(a.cu_q + lo);
    pos = t - q0;
    if (a.cu_k != nullptr)
      pos += static_cast<long long>(__ldg(a.cu_k + lo + 1) - __ldg(a.cu_k + lo)) -
             (__ldg(a.cu_q + lo + 1) - q0);
  }
  const float ratio = (static_cast<float>(pos) + 1.f) / a.nf;
  return 1.f + a.alpha * logf(fmaxf(ratio, 1.f));
}

// Quad q = tt * per_tile + rem, rem = hq * col_blocks + cb (heads 4 hq .. 4 hq + 3).
struct Cursor {
  long long u, tt;
  int rem;
};

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    rel_logits_kernel(const __grid_constant__ RelLogitsKernelArgs a,
                      const __grid_constant__ CUtensorMap tm_rel) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&s.mma_bar, 1);
    s.abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_rel);
  }
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;
  const AbortCtx ab{&s.abort_flag, a.status, kStatusRelLogitsTimeout};

  const int per_tile = a.head_quads * a.col_blocks;
  const long long step_tt = static_cast<long long>(gridDim.x) / per_tile;
  const int step_rem = static_cast<int>(gridDim.x - step_tt * per_tile);
  auto advance = [&](Cursor c) {
    c.u += gridDim.x;
    c.tt += step_tt;
    c.rem += step_rem;
    if (c.rem >= per_tile) {
      c.rem -= per_tile;
      ++c.tt;
    }
    return c;
  };
  auto quad_of = [&](int rem) { return a.col_blocks == 1 ? rem : rem / a.col_blocks; };

  const uint64_t adesc = sdesc_sw128(smem_u32(s.a), 16, 1024);
  const uint64_t bdesc = sdesc_sw128(smem_u32(s.b[0]), kBHalf, 1024);
  const uint32_t sw = static_cast<uint32_t>(tid & 7);
  uint8_t* const my_row = s.a + tid * 128;
  // Weight chunk of this thread: row j = tid / 8, columns 8 * (tid % 8) .. + 7 of each half.
  const int wj = tid >> 3;
  const int wq = tid & 7;
  const uint32_t b_off = static_cast<uint32_t>(wj * 128) +
                         ((static_cast<uint32_t>(wq) ^ static_cast<uint32_t>(wj & 7)) << 4);

  // This thread's r row of a quad: token tt * 128 + tid, heads 4 hq .. 4 hq + 3 (16 features
  // each); zeros past the last token and head.
  auto load_r = [&](const Cursor& c, uint4 (&x)[8]) {
    const long long t = c.tt * kRows + tid;
    const int h0 = 4 * quad_of(c.rem);
    const uint16_t* p = a.r + t * a.r_st + static_cast<long long>(h0) * a.r_sh;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const bool valid = t < a.total_q && h0 + k < a.n_heads;
      const uint16_t* pk = p + k * a.r_sh;
      x[2 * k] = valid ? ldg_nc_v4(pk) : make_uint4(0u, 0u, 0u, 0u);
      x[2 * k + 1] = valid ? ldg_nc_v4(pk + 8) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // This thread's weight chunk of head h, column block cb (both halves); zeros past rel_extent.
  auto load_w = [&](int h, int cb, uint4& x0, uint4& x1) {
    const int e0 = cb * kCols + wq * 8;
    const uint16_t* p = a.w + static_cast<long long>(h) * a.w_sh + wj * a.w_sj + e0;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    x0 = e0 < a.rel_extent ? ldg_nc_v4(p) : z;
    x1 = e0 + 64 < a.rel_extent ? ldg_nc_v4(p + 64) : z;
  };
  // Weight slice identity (a shared weight has one slice per column block).
  auto key_of = [&](int h, int cb) { return (a.w_sh != 0 ? h * a.col_blocks : 0) + cb; };

  Cursor cur;
  cur.u = blockIdx.x;
  cur.tt = cur.u / per_tile;
  cur.rem = static_cast<int>(cur.u - cur.tt * per_tile);
  uint4 rq[8];
  uint4 w0 = make_uint4(0u, 0u, 0u, 0u), w1 = w0;
  int w_key = -1;  // key of the weight chunk held in w0 / w1
  if (cur.u < a.units) {
    load_r(cur, rq);
    const int hq = quad_of(cur.rem);
    load_w(4 * hq, cur.rem - hq * a.col_blocks, w0, w1);
    w_key = key_of(4 * hq, cur.rem - hq * a.col_blocks);
  }
  int b_key = -1;  // key of the weight slice in shared memory
  uint32_t phase = 0;
  bool stop = false;
  while (cur.u < a.units && !stop) {
    const int hq = quad_of(cur.rem);
    const int cb = cur.rem - hq * a.col_blocks;
    const int nk_heads = min(4, a.n_heads - 4 * hq);
    const Cursor nxt = advance(cur);
    const float tau = row_tau(a, cur.tt * kRows + tid);
    const uint64_t tau2 = f2_pack(tau, tau);

    // The quad's r rows into shared memory.  The previous unit's MMA has completed (its barrier
    // was waited on), so the tile is free.
#pragma unroll
    for (int c = 0; c < 8; ++c) st_shared_v4(my_row + ((static_cast<uint32_t>(c) ^ sw) << 4), rq[c]);

    for (int k = 0; k < nk_heads; ++k) {
      const int h = 4 * hq + k;
      if (w_key != b_key) {  // CTA-uniform
        b_key = w_key;
        st_shared_v4(s.b[0] + b_off, w0);
        st_shared_v4(s.b[1] + b_off, w1);
      }
      fence_proxy_async_smem();
      if (tid == 0) bulk_wait_read_all();  // the staging tile's previous stores have read it
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        umma_ss(tbase, sdesc_advance(adesc, 32u * k), bdesc, kIdesc, 0u);
        umma_commit(&s.mma_bar);
      }

      // While the MMA runs: the next unit's weight chunk and, once per quad, the next quad's r.
      if (k + 1 < nk_heads) {
        const int nk = key_of(h + 1, cb);
        if (nk != w_key) {
          load_w(h + 1, cb, w0, w1);
          w_key = nk;
        }
      } else if (nxt.u < a.units) {
        const int nq = quad_of(nxt.rem);
        const int ncb = nxt.rem - nq * a.col_blocks;
        const int nk = key_of(4 * nq, ncb);
        if (nk != w_key) {
          load_w(4 * nq, ncb, w0, w1);
          w_key = nk;
        }
      }
      if (k == 0 && nxt.u < a.units) load_r(nxt, rq);

      const bool ok = mbar_wait_warp(&s.mma_bar, phase, ab);
      phase ^= 1u;
      if (__syncthreads_or(ok ? 0 : 1)) {
        stop = true;
        break;
      }
      tc_fence_after();

      const uint32_t trow = tbase + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll
      for (int c32 = 0; c32 < 4; ++c32) {
        uint32_t v[32];
        tmem_ld32(trow + c32 * 32, v);
        tmem_wait_ld();
        uint8_t* dst = s.out[c32 >> 1] + tid * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 8 * q + 2 * e;
            pk[e] = pack_bf16(f2_mul(f2_pack(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), tau2));
          }
          const uint32_t chunk = static_cast<uint32_t>((c32 & 1) * 4 + q);
          st_shared_v4(dst + ((chunk ^ sw) << 4), make_uint4(pk[0], pk[1], pk[2], pk[3]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        const int x0 = cb * kCols;
        const int y = static_cast<int>(cur.tt * kRows);
        tma_store_3d(&tm_rel, s.out[0], x0, h, y);
        if (x0 + 64 < a.rel_extent) tma_store_3d(&tm_rel, s.out[1], x0 + 64, h, y);
        bulk_commit_group();
      }
    }
    cur = nxt;
  }

  if (tid == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace rl

cudaError_t launch_rel_logits_sm100(const RelLogitsKernelArgs& args, const CUtensorMap& tm_rel,
                                    int grid, cudaStream_t stream) {
  static std::atomic<bool> attr_set[64];
  cudaError_t e = set_smem_limit_once(rl::rel_logits_kernel, rl::kSmemAlloc, attr_set);
  if (e != cudaSuccess) return e;
  rl::rel_logits_kernel<<<grid, rl::kThreads, rl::kSmemAlloc, stream>>>(args, tm_rel);
  return cudaGetLastError();
}

}  // namespace ifa4
