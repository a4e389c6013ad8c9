// FA4-style relative-bias flash-attention prefill for sm_100a (B200).
//
// One CTA owns two 128-row query sub-tiles that share a KV head ("ping-pong"): either two
// query heads of one GQA group at the same rows (even group size), or two consecutive 128-row
// blocks of one head.  Warp roles (12 warps, 384 threads; after set-up setmaxnreg leaves warps
// 0-3 56 registers each and gives the softmax warps 224):
//   warp 0      TMA producer: Q sub-tiles once per work tile, then K/V tiles through a
//               two-stage ring (128 keys x 128 dims, 128-byte swizzle, no multicast).
//   warp 1      UMMA issuer (one thread): S_s = Q_s K^T (SS, both K-major) into TMEM, then
//               O_s += P_s V (TS: P from TMEM, V MN-major) for s = 0, 1, interleaved so the
//               tensor core works on one sub-tile while the other one's softmax runs.
//   warp 2      owns the TMEM allocation (512 columns: S0 | S1 | O0 | O1).
//   warps 4-7   softmax of sub-tile 0, warps 8-11 softmax of sub-tile 1: one thread per
//               query row (= TMEM lane).  Scale, fused relative-bias gather, causal/window
//               mask, online softmax in the exp2 domain with conditional O rescaling (only
//               when the running max grows by more than 2^8), P written back to TMEM as bf16
//               over the first 64 columns of S, epilogue O / l -> bf16 -> global.
//
// Paged KV cache (kPaged): K/V come from [num_pages, page_size, kv_heads, 128] caches through
// a block table.  The whole of warp 0 produces: lanes fetch the page numbers of the next KV tile
// while the current one is issued, and each 128-key tile is loaded as 128 / box units of box =
// min(page_size, 128) rows, one 4-D TMA box per unit and 64-dim half, into the same swizzled
// layout as the contiguous path.  Units at or past the sequence's end load zeros (an
// out-of-range page coordinate).  The unit that holds the sequence's last key is copied into
// the V stage by the warp itself with its rows past the last key zeroed: P is 0 there, but a
// NaN left in an unused cache slot would still turn 0 * NaN into NaN in the P.V product
// (unused K rows are harmless: the mask replaces their scores).
//
// Causal and sliding-window masks prune KV tiles before any load: the loop covers exactly the
// tiles [j_lo, j_hi) that intersect the union of the two sub-tiles' visible key ranges; the
// per-element mask runs only for rows whose range does not cover the whole tile.
//
// Semantics: reference.py:27-39 (oracle) with the kernel-side conventions of
// triton_kernel.py:43-82 (rows with no visible key give 0, scale applies to QK^T only, the
// bias is added after scaling).  Bias distance d = q_pos + bias_shift - k_pos with
// bias_shift = sq - sk (reference alignment) or sk - sq (bottom-right); the mask diagonal is
// shifted by 0 (reference) or sk - sq (bottom-right).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ifa4_internal.h"
#include "ifa4_ptx.cuh"

namespace ifa4 {
namespace prefill {

constexpr int kBM = 128;                                 // query rows per sub-tile
constexpr int kBN = 128;                                 // keys per KV tile
constexpr int kThreads = 384;
// register split after set-up: warps 0-3 (producer, MMA issuer, TMEM owner) give registers to the
// eight softmax warps, 4 x 32 x 56 + 8 x 32 x 224 = 64512 = 384 threads x 168 at launch
constexpr int kRegsControl = 56, kRegsSoftmax = 224;
static_assert(4 * 32 * kRegsControl + 8 * 32 * kRegsSoftmax <= 384 * 168, "register split");
constexpr uint32_t kHalf = 128u * 128u;                  // 128 rows x 128 B (64 dims)
constexpr uint32_t kTile = 2u * kHalf;                   // 128 rows x 256 B (128 dims)
constexpr uint32_t kSmemQ = 0;                           // 2 sub-tiles
constexpr uint32_t kSmemK = 2 * kTile;                   // 2 stages
constexpr uint32_t kSmemV = 4 * kTile;                   // 2 stages
constexpr uint32_t kSmemBar = 6 * kTile;                 // barriers + slots
// Per softmax warp, a 32-row x 32-column bf16 transpose buffer for the relative-bias gather;
// rows are 34 halfwords (17 words) apart so both the row writes and the per-lane row reads are
// free of bank conflicts.
constexpr uint32_t kBiasRowHalves = 34;
constexpr uint32_t kBiasWarpBytes = 32 * kBiasRowHalves * 2;
constexpr uint32_t kSmemBias = kSmemBar + 256;
constexpr uint32_t kSmemBytes = kSmemBias + 8 * kBiasWarpBytes;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;       // slack for 1024-B alignment
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;                // log2 units: rescale O at 256x


constexpr uint32_t kIdescQK = idesc_bf16_f32(128, 128, /*b_mn_major=*/false);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, /*b_mn_major=*/true);

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2];
  uint64_t o_full[2], o_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

struct TileInfo {
  int n_kv;      // KV tiles to visit (0: every row of both sub-tiles sees no key)
  int j_lo;      // first KV tile
  int head[2];
  int row0[2];   // first local query row of each sub-tile
  int kvh;
};

__device__ __forceinline__ TileInfo tile_info(const PrefillKernelArgs& a, int qt, int hslot,
                                              int sq, int sk, bool split_on, int split) {
  TileInfo t;
  if (a.pair_heads) {
    t.head[0] = 2 * hslot;
    t.head[1] = 2 * hslot + 1;
    t.row0[0] = t.row0[1] = qt * kBM;
  } else {
    t.head[0] = t.head[1] = hslot;
    t.row0[0] = qt * 2 * kBM;
    t.row0[1] = qt * 2 * kBM + kBM;
  }
  t.kvh = t.head[0] / (a.n_heads / a.kv_heads);
  const int ms = a.align_bottom_right ? sk - sq : 0;
  int lo = 0x7fffffff, hi = -0x7fffffff;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int r0 = t.row0[s];
    if (r0 >= sq) continue;
    const int r1 = min(r0 + kBM, sq);
    int h = sk;
    if (a.causal) h = min(h, r1 + ms);
    int l = 0;
    if (a.window_left >= 0) l = max(0, r0 + ms - a.window_left);
    if (h > l) {
      lo = min(lo, l);
      hi = max(hi, h);
    }
  }
  if (hi <= lo) {
    t.n_kv = 0;
    t.j_lo = 0;
  } else {
    t.j_lo = lo / kBN;
    t.n_kv = (hi + kBN - 1) / kBN - t.j_lo;
  }
  if (split_on && t.n_kv > 0) {  // this CTA's share of the KV tiles: [first, first + n)
    const int per = (t.n_kv + a.kv_splits - 1) / a.kv_splits;
    const int first = split * per;
    t.j_lo += first;
    t.n_kv = max(0, min(per, t.n_kv - first));
  }
  return t;
}

// Producer for a paged KV cache: run by all 32 lanes of warp 0 (see the file comment).
template <bool kSplit>
__device__ __forceinline__ void produce_paged(const PrefillKernelArgs& a, uint8_t* smem,
                                              Bars* bars, const CUtensorMap* tm_q,
                                              const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                              int hslot, int b, int q_start, int sq, int sk,
                                              int n_qt, int slot0, int slot_step, int split,
                                              int lane, const AbortCtx& ab) {
  uint32_t qc = 0, kc = 0, vc = 0;
  const uint64_t pol_kv = l2_policy_evict_last();
  const uint64_t pol_q = l2_policy_evict_first();
  const int box = 1 << a.box_shift;
  const int units = kBN >> a.box_shift;
  const int page_mask = (1 << a.page_shift) - 1;
  const int32_t* bt = a.block_table + static_cast<long long>(b) * a.bt_stride;
  bool ok = true;
  for (int slot = slot0; slot < n_qt && ok; slot += slot_step) {
    const TileInfo t = tile_info(a, n_qt - 1 - slot, hslot, sq, sk, kSplit, split);
    if (t.n_kv == 0) continue;
    if (!(ok = mbar_wait_warp(&bars->q_empty, (qc & 1) ^ 1, ab))) break;
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->q_full, 2 * kTile);
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d_hint(smem + kSmemQ + s * kTile + hf * kHalf, tm_q, &bars->q_full, hf * 64,
                           t.head[s], q_start + t.row0[s], pol_q);
    }
    ++qc;
    // page of unit `lane` of KV tile j; -1 past the sequence's end or for an entry outside
    // [0, num_pages)
    auto unit_block = [&](int j) {
      const int key = (t.j_lo + j) * kBN + lane * box;
      int blk = -1;
      if (lane < units && key < sk) {
        blk = __ldg(bt + (key >> a.page_shift));
        if (blk < 0 || blk >= a.num_pages) blk = -1;
      }
      return blk;
    };
    int blk = unit_block(0);
    for (int j = 0; j < t.n_kv; ++j) {
      const int key0 = (t.j_lo + j) * kBN;
      const int blk_next = j + 1 < t.n_kv ? unit_block(j + 1) : -1;  // in flight across waits
      const int in_page = (key0 + lane * box) & page_mask;
      const int page = blk >= 0 ? blk : a.num_pages;  // out of range: TMA writes zeros
      const uint32_t ks = kc & 1;
      if (!(ok = mbar_wait_warp(&bars->k_empty[ks], ((kc >> 1) & 1) ^ 1, ab))) break;
      if (lane == 0) mbar_arrive_expect_tx(&bars->k_full[ks], kTile);
      __syncwarp();
      if (lane < units) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          tma_load_4d_hint(smem + kSmemK + ks * kTile + hf * kHalf + lane * box * 128, tm_k,
                           &bars->k_full[ks], hf * 64, t.kvh, in_page, page, pol_kv);
      }
      ++kc;
      const uint32_t vs = vc & 1;
      if (!(ok = mbar_wait_warp(&bars->v_empty[vs], ((vc >> 1) & 1) ^ 1, ab))) break;
      // the unit holding the sequence's last key, unless that key ends the unit
      const int pu = (key0 < sk && sk < key0 + kBN && (sk & (box - 1)) != 0)
                         ? (sk - key0) >> a.box_shift : -1;
      uint32_t v_bytes = kTile;
      if (pu >= 0) {
        const int pblk = __shfl_sync(0xffffffffu, blk, pu);
        IFA4_DBG_CHECK(a.status, pblk < a.num_pages);
        const int pkey = key0 + pu * box;
        const int nvalid = sk - pkey;
        const uint16_t* src = a.v + static_cast<long long>(pblk < 0 ? 0 : pblk) * a.v_sp +
                              static_cast<long long>(pkey & page_mask) * a.v_st +
                              static_cast<long long>(t.kvh) * a.v_sh;
        uint8_t* dst = smem + kSmemV + vs * kTile;
#pragma unroll 4
        for (int i = lane; i < box * 16; i += 32) {
          const int r = i >> 4, ch = i & 15;
          uint4 val = make_uint4(0u, 0u, 0u, 0u);
          if (r < nvalid && pblk >= 0) val = ldg_nc_v4(src + static_cast<long long>(r) * a.v_st + ch * 8);
          const int row = pu * box + r;
          *reinterpret_cast<uint4*>(dst + (ch >> 3) * kHalf + row * 128 +
                                    (((ch & 7) ^ (row & 7)) << 4)) = val;
        }
        fence_proxy_async_smem();  // the UMMA reads these bytes through the async proxy
        __syncwarp();
        v_bytes -= static_cast<uint32_t>(box) * 256u;
      }
      if (lane == 0) mbar_arrive_expect_tx(&bars->v_full[vs], v_bytes);
      __syncwarp();
      if (lane < units && lane != pu) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          tma_load_4d_hint(smem + kSmemV + vs * kTile + hf * kHalf + lane * box * 128, tm_v,
                           &bars->v_full[vs], hf * 64, t.kvh, in_page, page, pol_kv);
      }
      ++vc;
      blk = blk_next;
    }
  }
  // Drain: every issued load has completed before the CTA may exit.
  if (lane == 0) {
    if (qc > 0) mbar_wait(&bars->q_full, (qc - 1) & 1, ab);
    for (uint32_t i = 0; i < 2 && i < kc; ++i) {
      const uint32_t last = kc - 1 - i;
      mbar_wait(&bars->k_full[last & 1], (last >> 1) & 1, ab);
    }
    for (uint32_t i = 0; i < 2 && i < vc; ++i) {
      const uint32_t last = vc - 1 - i;
      mbar_wait(&bars->v_full[last & 1], (last >> 1) & 1, ab);
    }
  }
}

__device__ __forceinline__ void issue_qk(uint32_t tmem_s, uint32_t q_addr, uint32_t k_addr) {
  const uint64_t qd = sdesc_sw128(q_addr, 16, 1024);
  const uint64_t kd = sdesc_sw128(k_addr, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
    umma_ss(tmem_s, sdesc_advance(qd, off), sdesc_advance(kd, off), kIdescQK, kk > 0 ? 1u : 0u);
  }
}

__device__ __forceinline__ void issue_pv(uint32_t tmem_o, uint32_t tmem_p, uint32_t v_addr,
                                         bool accumulate) {
  const uint64_t vd = sdesc_sw128(v_addr, kHalf, 1024);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    umma_ts(tmem_o, tmem_p + kk * 8, sdesc_advance(vd, kk * 2048), kIdescPV,
            (kk > 0 || accumulate) ? 1u : 0u);
  }
}

template <int kEmu, int kHalf2, bool kPaged, bool kPeers, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
    rel_attn_prefill_kernel(const __grid_constant__ PrefillKernelArgs a,
                            const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kSmemBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Grid (query slots, head slots, sequences) when one query tile's key range over all KV
  // heads outgrows L2: the query slots of one head slot then launch together, so the CTAs
  // resident at one time read the K/V of few KV heads and those tiles stay in L2.  Otherwise
  // (head slots, sequences, query slots), which spreads a ragged batch's sequences over the
  // first waves.
  // The slot dimension carries the query slot and, for a split launch, the KV split (fastest).
  const int hslot = a.q_fastest ? blockIdx.y : blockIdx.x;
  const int b = a.q_fastest ? blockIdx.z : blockIdx.y;
  const int slot_idx = a.q_fastest ? blockIdx.x : blockIdx.z;
  const int nsplit = kSplit ? a.kv_splits : 1;
  const int split = slot_idx % nsplit;
  const int slot0 = slot_idx / nsplit;
  const int slot_step = (a.q_fastest ? gridDim.x : gridDim.z) / nsplit;
  const int q_start = a.cu_q[b];
  const int sq = a.cu_q[b + 1] - q_start;
  const int k_start = a.cu_k[b];
  const int sk = a.cu_k[b + 1] - k_start;
  const int rows_per_cta = a.pair_heads ? kBM : 2 * kBM;
  const int n_qt = (sq + rows_per_cta - 1) / rows_per_cta;
  if (slot0 >= n_qt) return;  // uniform over the CTA: nothing to do

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1 + 8);  // MMA commit + 8 softmax warps (epilogue staging)
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 4);   // one arrival per softmax warp
      mbar_init(&bars->o_full[i], 1);
      mbar_init(&bars->o_empty[i], 4);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const AbortCtx ab{&bars->abort_flag, a.status, kStatusPrefillTimeout};
  if (warp < 4) setmaxnreg_dec<kRegsControl>();
  else setmaxnreg_inc<kRegsSoftmax>();
  if (warp < 4) {
   if (kPaged && warp == 0) {
    produce_paged<kSplit>(a, smem, bars, &tm_q, &tm_k, &tm_v, hslot, b, q_start, sq, sk, n_qt,
                          slot0, slot_step, split, lane, ab);
   } else if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t qc = 0, kc = 0, vc = 0;
      const uint64_t pol_kv = l2_policy_evict_last();
      const uint64_t pol_q = l2_policy_evict_first();
      for (int slot = slot0; slot < n_qt; slot += slot_step) {
        const TileInfo t = tile_info(a, n_qt - 1 - slot, hslot, sq, sk, kSplit, split);
        if (t.n_kv == 0) continue;
        if (!mbar_wait(&bars->q_empty, (qc & 1) ^ 1, ab)) break;
        mbar_arrive_expect_tx(&bars->q_full, 2 * kTile);
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d_hint(smem + kSmemQ + s * kTile + hf * kHalf, &tm_q, &bars->q_full,
                             hf * 64, t.head[s], q_start + t.row0[s], pol_q);
        ++qc;
        bool ok = true;
        for (int j = 0; j < t.n_kv && ok; ++j) {
          const int row = k_start + (t.j_lo + j) * kBN;
          const uint32_t ks = kc & 1;
          if (!(ok = mbar_wait(&bars->k_empty[ks], ((kc >> 1) & 1) ^ 1, ab))) break;
          mbar_arrive_expect_tx(&bars->k_full[ks], kTile);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d_hint(smem + kSmemK + ks * kTile + hf * kHalf, &tm_k, &bars->k_full[ks],
                             hf * 64, t.kvh, row, pol_kv);
          ++kc;
          const uint32_t vs = vc & 1;
          if (!(ok = mbar_wait(&bars->v_empty[vs], ((vc >> 1) & 1) ^ 1, ab))) break;
          mbar_arrive_expect_tx(&bars->v_full[vs], kTile);
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d_hint(smem + kSmemV + vs * kTile + hf * kHalf, &tm_v, &bars->v_full[vs],
                             hf * 64, t.kvh, row, pol_kv);
          ++vc;
        }
        if (!ok) break;
      }
      // Drain: every issued load has completed before the CTA may exit (the full barrier of
      // the last use of each stage has passed that phase once the bytes landed).
      if (qc > 0) mbar_wait(&bars->q_full, (qc - 1) & 1, ab);
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
      uint32_t qc = 0, kc = 0, vc = 0, pc = 0, oc = 0;
      const uint32_t q_addr = smem_u32(smem + kSmemQ);
      const uint32_t k_addr = smem_u32(smem + kSmemK);
      const uint32_t v_addr = smem_u32(smem + kSmemV);
      bool ok = true;
      for (int slot = slot0; slot < n_qt && ok; slot += slot_step) {
        const TileInfo t = tile_info(a, n_qt - 1 - slot, hslot, sq, sk, kSplit, split);
        if (t.n_kv == 0) continue;
        if (!(ok = mbar_wait(&bars->q_full, qc & 1, ab))) break;
        ++qc;
        // first KV tile: S_s = Q_s K^T
        uint32_t ks = kc & 1;
        if (!(ok = mbar_wait(&bars->k_full[ks], (kc >> 1) & 1, ab))) break;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          issue_qk(tbase + s * 128, q_addr + s * kTile, k_addr + ks * kTile);
          umma_commit(&bars->s_full[s]);
        }
        umma_commit(&bars->k_empty[ks]);
        ++kc;
        for (int j = 1; j < t.n_kv && ok; ++j) {
          ks = kc & 1;
          const uint32_t vs = vc & 1;
          if (!(ok = mbar_wait(&bars->k_full[ks], (kc >> 1) & 1, ab))) break;
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            if (!(ok = mbar_wait(&bars->p_full[s], pc & 1, ab))) break;
            if (j == 1 && !(ok = mbar_wait(&bars->o_empty[s], (oc & 1) ^ 1, ab))) break;
            if (s == 0 && !(ok = mbar_wait(&bars->v_full[vs], (vc >> 1) & 1, ab))) break;
            tc_fence_after();
            issue_pv(tbase + 256 + s * 128, tbase + s * 128, v_addr + vs * kTile, j > 1);
            issue_qk(tbase + s * 128, q_addr + s * kTile, k_addr + ks * kTile);
            umma_commit(&bars->s_full[s]);
          }
          if (!ok) break;
          ++pc;
          umma_commit(&bars->k_empty[ks]);
          ++kc;
          umma_commit(&bars->v_empty[vs]);
          ++vc;
        }
        if (!ok) break;
        // last KV tile: O_s += P_s V
        const uint32_t vs = vc & 1;
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          if (!(ok = mbar_wait(&bars->p_full[s], pc & 1, ab))) break;
          if (t.n_kv == 1 && !(ok = mbar_wait(&bars->o_empty[s], (oc & 1) ^ 1, ab))) break;
          if (s == 0 && !(ok = mbar_wait(&bars->v_full[vs], (vc >> 1) & 1, ab))) break;
          tc_fence_after();
          issue_pv(tbase + 256 + s * 128, tbase + s * 128, v_addr + vs * kTile, t.n_kv > 1);
          umma_commit(&bars->o_full[s]);
        }
        if (!ok) break;
        ++pc;
        umma_commit(&bars->v_empty[vs]);
        ++vc;
        umma_commit(&bars->q_empty);
        ++oc;
      }
      // Drain: all issued MMAs complete before TMEM is released.
      umma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, ab);
    }
   }
  } else {
    // ------------------------------------------------------------------ softmax
    const int s = (warp - 4) >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tbase + lane_off + s * 128;
    const uint32_t t_o = tbase + lane_off + 256 + s * 128;
    const int ms = a.align_bottom_right ? sk - sq : 0;
    const int bs = a.align_bottom_right ? sk - sq : sq - sk;
    uint32_t pc = 0, oc = 0;
    bool ok = true;
    for (int slot = slot0; slot < n_qt && ok; slot += slot_step) {
      const TileInfo t = tile_info(a, n_qt - 1 - slot, hslot, sq, sk, kSplit, split);
      const int qi = t.row0[s] + row;
      const bool row_valid = qi < sq;
      const int h = t.head[s];
      uint16_t* out_row = a.out + static_cast<long long>(q_start + qi) * a.out_st +
                          static_cast<long long>(h) * a.out_sh;
      if (t.n_kv == 0) {
        if (row_valid) {
          if (kSplit) {  // an empty share: its partial carries no weight in the merge
            if (IFA4_DBG_CHECK(a.status, split < a.kv_splits && q_start + qi < a.total_q))
              a.ws_lse[(static_cast<long long>(split) * a.n_heads + h) * a.total_q + q_start + qi] =
                -INFINITY;
          } else if (IFA4_DBG_CHECK(a.status, q_start + qi < a.total_q && h < a.n_heads)) {
            uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int c = 0; c < 16; ++c) reinterpret_cast<uint4*>(out_row)[c] = z;
            if (a.lse != nullptr)
              a.lse[static_cast<long long>(h) * a.lse_sh +
                    static_cast<long long>(q_start + qi) * a.lse_st] = -INFINITY;
          }
        }
        continue;
      }
      // report only (TMA loads outside a tensor read zeros, and rows past the sequence end are
      // never stored): the visited KV tiles start inside the sequence, the row inside the batch
      IFA4_DBG_CHECK(a.status, t.j_lo >= 0 && (t.j_lo + t.n_kv - 1) * kBN < sk &&
                                   (!row_valid || q_start + qi < a.total_q));
      const uint16_t* rel_row = a.rel + static_cast<long long>(q_start + qi) * a.rel_st +
                                static_cast<long long>(h) * a.rel_sh;
      // visible keys of this row: [key_lo, key_hi)
      int key_hi = sk;
      if (a.causal) key_hi = min(key_hi, qi + ms + 1);
      const int key_lo = a.window_left >= 0 ? max(0, qi + ms - a.window_left) : 0;
      const int dmax = qi + bs;  // bias distance at key 0
      // The band tiles (those whose distances meet [0, R)) come last in the KV loop; start
      // pulling this row's bias into L2 now so their gather finds it there.
      if (row_valid) {  // addresses stay inside the row's R elements
        const int n = min((a.rel_extent + 63) / 64, 16);
        for (int i = 0; i < n; ++i) prefetch_l2(rel_row + i * 64);
      }
      uint16_t* bias_buf = reinterpret_cast<uint16_t*>(smem + kSmemBias + (warp - 4) * kBiasWarpBytes);
      float m_run = -INFINITY, l_run = 0.f;

      for (int j = 0; j < t.n_kv; ++j) {
        const int k0 = (t.j_lo + j) * kBN;
        // relative bias: keys in [dmax - R + 1, dmax] carry rel[row, dmax - key]
        const int bl = dmax - a.rel_extent + 1 - k0;  // first column with bias
        const int bh = dmax - k0;                     // last column with bias
        const int cl = key_lo - k0, ch = key_hi - k0;  // visible columns [cl, ch)
        const bool has_bias = row_valid && bl <= 127 && bh >= 0;
        const bool has_mask = cl > 0 || ch < kBN;
        const bool warp_bias = __any_sync(0xffffffffu, has_bias);
        // Vector bias path: the first two chunks' windows are loaded before S arrives, so their
        // round trip overlaps the wait; chunk c + 2 is loaded when chunk c has been used.
        uint32_t bwin[2][20];
        if (a.bias_vec && warp_bias) {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
            load_bias_window(rel_row, bh, cc, a.rel_extent,
                             has_bias && cc * 32 + 31 >= bl && cc * 32 <= bh, bwin[cc]);
        }
        if (!(ok = mbar_wait_warp(&bars->s_full[s], pc & 1, ab))) break;
        ++pc;
        tc_fence_after();
        // Interior tiles after the first: the exponentials are taken against the running max
        // m_run without a row-max pass.  A score above m_run only makes its p larger than 1,
        // which fp32 sums and bf16 P hold exactly as well up to 2^32; the tile's sum of p shows
        // whether any went past that (or overflowed).  P stays in registers until then, so if
        // one did, S is still intact in TMEM and the two passes below redo the tile with its
        // true max (rescaling O and l as usual).
        bool done = false;
        if (j > 0 && !__any_sync(0xffffffffu, has_bias || has_mask)) {
          const uint64_t mul2 = f2_pack(a.scale_log2, a.scale_log2);
          const uint64_t neg2 = f2_pack(-m_run, -m_run);
          uint64_t acc[4] = {0, 0, 0, 0};
          uint32_t pk[2][32];
          uint32_t rq[2][16];
          tmem_ld16(t_s, rq[0]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            if (c < 7) tmem_ld16(t_s + (c + 1) * 16, rq[(c + 1) & 1]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int col = c * 16 + 2 * i;
              float y0, y1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(rq[c & 1][2 * i]),
                                       __uint_as_float(rq[c & 1][2 * i + 1])),
                               mul2, neg2),
                        y0, y1);
              float p0, p1;
              if ((col & 15) < kEmu) {
                exp2_poly_pair_capped(y0, y1, p0, p1);
              } else if ((col & 15) < kEmu + kHalf2) {
                exp2_h2_pair(y0, y1, p0, p1);  // fp16: >= 2^16 is inf, caught below
              } else {
                p0 = fast_exp2(y0);
                p1 = fast_exp2(y1);
              }
              acc[i & 3] = f2_add(acc[i & 3], f2_pack(p0, p1));
              pk[c >> 2][(c & 3) * 8 + i] = pack_bf16x2(p0, p1);
            }
            if (c < 7) tmem_wait_ld();
          }
          const uint64_t a01 = f2_add(acc[0], acc[1]), a23 = f2_add(acc[2], acc[3]);
          float u0, u1;
          f2_unpack(f2_add(a01, a23), u0, u1);
          const float l_tile = u0 + u1;
          if (__all_sync(0xffffffffu, l_tile <= 4294967296.0f)) {  // false for inf and NaN
            tmem_st32(t_s, pk[0]);
            tmem_st32(t_s + 32, pk[1]);
            l_run += l_tile;
            done = true;
          }
        }
        if (!done) {
          // Pass 1 — the row max.  In a warp where no row needs bias or mask it is taken over the
          // raw scores and the scale is folded into the exponent FMA (mul = scale*log2e).
          // Otherwise every lane turns its scores into the scaled, biased, masked logit chunk by
          // chunk and writes it back over S in TMEM, and pass 2 reads logits (mul = 1).
          // Score chunk 0 (columns 0..31) is pass 2's first operand: in interior warps pass 1
          // leaves it in rr[0], so pass 2 starts without a TMEM round trip.
          uint32_t rr[2][32];
          float mul, m_tile;
          if (!__any_sync(0xffffffffu, has_bias || has_mask)) {
            uint32_t r[3][32];  // score chunks 1..3
            tmem_ld32(t_s, rr[0]);
#pragma unroll
            for (int c = 0; c < 3; ++c) tmem_ld32(t_s + (c + 1) * 32, r[c]);
            tmem_wait_ld();
            auto col = [&](int c) -> float {
              return __uint_as_float(c < 32 ? rr[0][c] : r[(c >> 5) - 1][c & 31]);
            };
            // columns 0..3 start four chains, then 4..123 in steps of 8, then 124..127
            float mA = col(0), mB = col(1), mC = col(2), mD = col(3);
#pragma unroll
            for (int c = 4; c < 124; c += 8) {
              mA = fmax3(mA, col(c), col(c + 1));
              mB = fmax3(mB, col(c + 2), col(c + 3));
              mC = fmax3(mC, col(c + 4), col(c + 5));
              mD = fmax3(mD, col(c + 6), col(c + 7));
            }
            mA = fmax3(mA, col(124), col(125));
            mB = fmax3(mB, col(126), col(127));
            mul = a.scale_log2;
            m_tile = fmax3(mA, mB, fmaxf(mC, mD)) * mul;
          } else {
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
              tmem_ld32(t_s + c * 32, r);
              tmem_wait_ld();
              float x[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(r[i]) * a.scale_log2;
              // Relative bias, gathered by the whole warp: for each of the warp's 32 rows the
              // lanes load that row's 32 consecutive values (one coalesced 64-byte access),
              // store them to the transpose buffer, and each lane then reads its own row.
              // Columns outside [bl, bh] (or rows without bias) read 0.
              const bool chunk_bias = has_bias && c * 32 + 31 >= bl && c * 32 <= bh;
              if (a.bias_vec) {
                if (__any_sync(0xffffffffu, chunk_bias)) add_bias_window(bwin[c & 1], bh, c, x);
                if (c < 2 && warp_bias)
                  load_bias_window(rel_row, bh, c + 2, a.rel_extent,
                                   has_bias && (c + 2) * 32 + 31 >= bl && (c + 2) * 32 <= bh,
                                   bwin[c & 1]);
              } else if (__any_sync(0xffffffffu, chunk_bias)) {
                uint16_t* buf = bias_buf;
                const int col = c * 32 + lane;
                uint16_t v[32];
#pragma unroll
                for (int tr = 0; tr < 32; ++tr) {  // all 32 loads in flight before any use
                  const int qi_t = qi - lane + tr;  // row of lane tr in this warp
                  const int d = qi_t + bs - k0 - col;
                  v[tr] = 0;
                  if (qi_t < sq && d >= 0 && d < a.rel_extent)
                    v[tr] = __ldg(rel_row + static_cast<long long>(tr - lane) * a.rel_st + d);
                }
#pragma unroll
                for (int tr = 0; tr < 32; ++tr) buf[tr * kBiasRowHalves + lane] = v[tr];
                __syncwarp();
                const uint32_t* w = reinterpret_cast<const uint32_t*>(buf) + lane * (kBiasRowHalves / 2);
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                  const uint32_t pr = w[k];
                  x[2 * k] += __uint_as_float(pr << 16) * kLog2e;
                  x[2 * k + 1] += __uint_as_float(pr & 0xffff0000u) * kLog2e;
                }
                __syncwarp();
              }
              if (has_mask) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  const int col = c * 32 + i;
                  if (col < cl || col >= ch) x[i] = -INFINITY;
                }
              }
              float m0 = x[0], m1 = x[1];
#pragma unroll
              for (int i = 2; i < 30; i += 4) {  // columns 2..29, then 30 and 31
                m0 = fmax3(m0, x[i], x[i + 1]);
                m1 = fmax3(m1, x[i + 2], x[i + 3]);
              }
              m0 = fmax3(m0, x[30], x[31]);
              mx = fmax3(mx, m0, m1);
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(x[i]);
              __syncwarp();  // reconverge after the per-row branches: tcgen05.st is .aligned
              tmem_st32(t_s + c * 32, r);
            }
            tmem_wait_st();  // pass 2 reads these columns back
            tmem_ld32(t_s, rr[0]);
            tmem_wait_ld();
            mul = 1.f;
            m_tile = mx;
          }
          const float m_new = fmaxf(m_run, m_tile);
          float alpha = 1.f;
          bool need_rescale = false;
          if (j == 0) {
            m_run = m_new;
          } else if (m_new > m_run + kRescaleThreshold) {
            alpha = fast_exp2(m_run - m_new);
            need_rescale = true;
            l_run *= alpha;
            m_run = m_new;
          }
          const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
          __syncwarp();  // reconverge: the tcgen05 operations below are .sync.aligned
          // Pass 2 — p = 2^(x * mul - m_use) over 32-column chunks (chunk 0 already in rr[0]),
          // loading chunk c+1 while chunk c is computed.  All exponentials on the SFU in fp32
          // (this path carries the masked tiles, whose -inf logits must give exactly 0; the
          // FMA-pipe and f16x2 variants apply to the single-pass interior path above).  P (bf16
          // pairs) goes to TMEM columns [16c, 16c+16), which chunks c+1.. (columns >= 32(c+1))
          // never overlap.
          const uint64_t mul2 = f2_pack(mul, mul);
          const uint64_t neg2 = f2_pack(-m_use, -m_use);
          uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c < 3) tmem_ld32(t_s + (c + 1) * 32, rr[(c + 1) & 1]);
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float y0, y1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(rr[c & 1][2 * i]),
                                       __uint_as_float(rr[c & 1][2 * i + 1])),
                               mul2, neg2),
                        y0, y1);
              const float p0 = fast_exp2(y0), p1 = fast_exp2(y1);
              acc[i & 3] = f2_add(acc[i & 3], f2_pack(p0, p1));
              pk[i] = pack_bf16x2(p0, p1);
            }
            tmem_st16(t_s + c * 16, pk);
            if (c < 3) tmem_wait_ld();
          }
          {
            const uint64_t a01 = f2_add(acc[0], acc[1]), a23 = f2_add(acc[2], acc[3]);
            float u0, u1;
            f2_unpack(f2_add(a01, a23), u0, u1);
            l_run += u0 + u1;
          }
          // Conditional O correction (PV of the previous tile is complete: its commit
          // preceded this tile's S commit).
          if (__any_sync(0xffffffffu, need_rescale)) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t o[32];
              tmem_ld32(t_o + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st32(t_o + c * 32, o);
            }
          }
        }
        // every lane's TMEM stores are complete and fenced before lane 0 releases P
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[s]);
      }
      if (!ok) break;
      // epilogue: O / l -> bf16, staged through this sub-tile's Q buffer (idle once O is final:
      // every MMA reading Q completed before the last PV) with the 128-B swizzle, then written
      // back by the warp as whole 256-byte rows (coalesced).  The producer reloads Q only after
      // the MMA commit and all 8 softmax warps have arrived on q_empty.
      if (!(ok = mbar_wait_warp(&bars->o_full[s], oc & 1, ab))) break;
      ++oc;
      tc_fence_after();
      // a row that never saw a visible key outputs 0 (its running max is still -inf)
      const bool seen = l_run > 0.f && m_run != -INFINITY;
      const float inv_l = seen ? 1.f / l_run : 0.f;
      if (!kSplit && a.lse != nullptr && row_valid &&  // ln(sum exp) = ln2 (m + log2 l)
          IFA4_DBG_CHECK(a.status, q_start + qi < a.total_q && h < a.n_heads))
        a.lse[static_cast<long long>(h) * a.lse_sh + static_cast<long long>(q_start + qi) * a.lse_st] =
            seen ? (m_run + __log2f(l_run)) * 0.6931471805599453f : -INFINITY;
      uint8_t* stage = smem + kSmemQ + s * kTile;
      if (kSplit) {
        // normalised fp32 partial (two 64-column halves, each staged through the Q buffer as
        // whole 256-byte row segments) and its log2-sum-exp, for the merge kernel
        if (row_valid && IFA4_DBG_CHECK(a.status, split < a.kv_splits && q_start + qi < a.total_q))
          a.ws_lse[(static_cast<long long>(split) * a.n_heads + h) * a.total_q + q_start + qi] =
              seen ? m_run + __log2f(l_run) : -INFINITY;
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
          __syncwarp();  // the previous half's reads of the stage are done
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + hp * 64 + c * 32, o);
            tmem_wait_ld();
            if (hp == 1 && c == 1) {  // TMEM O may be overwritten by the next work tile
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&bars->o_empty[s]);
            }
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const int g = c * 8 + v;  // 16-byte granule (4 floats) of the 256-byte segment
              uint4* dst = reinterpret_cast<uint4*>(stage + (g >> 3) * kHalf + row * 128 +
                                                    (((g & 7) ^ (row & 7)) << 4));
              *dst = make_uint4(__float_as_uint(__uint_as_float(o[4 * v]) * inv_l),
                                __float_as_uint(__uint_as_float(o[4 * v + 1]) * inv_l),
                                __float_as_uint(__uint_as_float(o[4 * v + 2]) * inv_l),
                                __float_as_uint(__uint_as_float(o[4 * v + 3]) * inv_l));
            }
          }
          __syncwarp();
          const int wrow0 = (warp & 3) * 32;
          const int g = lane & 15;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int r = wrow0 + 2 * i + (lane >> 4);
            const uint4 val = *reinterpret_cast<const uint4*>(
                stage + (g >> 3) * kHalf + r * 128 + (((g & 7) ^ (r & 7)) << 4));
            const int qr = t.row0[s] + r;
            if (qr < sq && IFA4_DBG_CHECK(a.status, q_start + qr < a.total_q))
              *reinterpret_cast<uint4*>(
                  a.ws_o + ((static_cast<long long>(split) * a.total_q + q_start + qr) * a.n_heads +
                            h) * 128 + hp * 64 + g * 4) = val;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->q_empty);
        continue;
      }
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(t_o + c * 32, o);
        tmem_wait_ld();
        if (c == 3) {  // TMEM O may be overwritten by the next work tile
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->o_empty[s]);
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv_l,
                              __uint_as_float(o[2 * i + 1]) * inv_l);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int g = c * 4 + v;  // 16-byte granule of the 256-byte row
          uint4* dst = reinterpret_cast<uint4*>(stage + (g >> 3) * kHalf + row * 128 +
                                                (((g & 7) ^ (row & 7)) << 4));
          *dst = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      __syncwarp();
      {
        const int wrow0 = (warp & 3) * 32;
        const int g = lane & 15;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int r = wrow0 + 2 * i + (lane >> 4);
          const uint4 val = *reinterpret_cast<const uint4*>(
              stage + (g >> 3) * kHalf + r * 128 + (((g & 7) ^ (r & 7)) << 4));
          const int qr = t.row0[s] + r;
          if (qr < sq && IFA4_DBG_CHECK(a.status, q_start + qr < a.total_q && h < a.n_heads)) {
            uint16_t* dst = a.out + static_cast<long long>(q_start + qr) * a.out_st +
                            static_cast<long long>(h) * a.out_sh + g * 8;
            *reinterpret_cast<uint4*>(dst) = val;
            if (kPeers) {  // the same row in other GPUs' outputs
              for (int pr = 0; pr < a.n_out_peers; ++pr)
                *reinterpret_cast<uint4*>(dst + a.out_peer_delta[pr]) = val;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->q_empty);
    }
  }

  // stores to other GPUs' outputs are performed system-wide before the CTA retires
  if (kPeers && warp >= 4) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// Merge of a split launch's partials, one warp per (token, head): weights 2^(lse_s - max lse)
// over the splits that saw a key; lanes own 4 of the 128 dims (16-byte loads, 8-byte stores).
__global__ void __launch_bounds__(256)
    rel_attn_prefill_combine_kernel(const __grid_constant__ PrefillKernelArgs a) {
  const long long w = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= a.total_q * a.n_heads) return;
  const long long t = w / a.n_heads;
  const int h = static_cast<int>(w % a.n_heads);
  const int S = a.kv_splits;
  if (!IFA4_DBG_CHECK(a.status, S >= 2 && S <= 16 && a.ws_o != nullptr && a.ws_lse != nullptr))
    return;
  float M = -INFINITY;
  for (int sp = 0; sp < S; ++sp)
    M = fmaxf(M, a.ws_lse[(static_cast<long long>(sp) * a.n_heads + h) * a.total_q + t]);
  float wsum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M != -INFINITY) {
    for (int sp = 0; sp < S; ++sp) {
      const float l = a.ws_lse[(static_cast<long long>(sp) * a.n_heads + h) * a.total_q + t];
      if (l == -INFINITY) continue;  // an empty share (its partial was never written)
      const float wt = fast_exp2(l - M);
      const float4 o = reinterpret_cast<const float4*>(
          a.ws_o + ((static_cast<long long>(sp) * a.total_q + t) * a.n_heads + h) * 128)[lane];
      wsum += wt;
      acc.x += wt * o.x;
      acc.y += wt * o.y;
      acc.z += wt * o.z;
      acc.w += wt * o.w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  uint2 packed;
  packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(a.out + t * a.out_st + static_cast<long long>(h) * a.out_sh +
                            lane * 4) = packed;
  if (lane == 0 && a.lse != nullptr)  // log2-sum-exp of the partials -> natural log
    a.lse[static_cast<long long>(h) * a.lse_sh + t * a.lse_st] =
        wsum > 0.f ? (M + __log2f(wsum)) * 0.6931471805599453f : -INFINITY;
}

}  // namespace prefill

namespace {
template <int kEmu, int kHalf2, bool kPaged, bool kPeers = false, bool kSplit = false>
cudaError_t launch_variant(const PrefillKernelArgs& args, const CUtensorMap& tm_q,
                           const CUtensorMap& tm_k, const CUtensorMap& tm_v, dim3 grid,
                           cudaStream_t stream) {
  static std::atomic<bool> attr_set[64];
  cudaError_t e =
      set_smem_limit_once(prefill::rel_attn_prefill_kernel<kEmu, kHalf2, kPaged, kPeers, kSplit>,
                          prefill::kSmemAlloc, attr_set);
  if (e != cudaSuccess) return e;
  prefill::rel_attn_prefill_kernel<kEmu, kHalf2, kPaged, kPeers, kSplit>
      <<<grid, prefill::kThreads, prefill::kSmemAlloc, stream>>>(args, tm_q, tm_k, tm_v);
  return cudaGetLastError();
}
}  // namespace

// tile_config -> (columns of 16 on the FMA-pipe polynomial, columns of 16 on SFU f16x2)
static const int kVariants[kPrefillNumTileConfigs][2] = {
    {kPrefillDefaultEmu, kPrefillDefaultHalf2}, {0, 0}, {2, 0}, {4, 0}, {6, 0}, {8, 0},
    {0, 16}, {0, 8}, {4, 8}};

cudaError_t launch_prefill_combine_sm100(const PrefillKernelArgs& args, cudaStream_t stream) {
  const long long pairs = args.total_q * args.n_heads;
  const long long blocks = (pairs + 7) / 8;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  prefill::rel_attn_prefill_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(args);
  return cudaGetLastError();
}

bool prefill_paged_tile_config_ok(int tile_config) {
  return tile_config >= 0 && tile_config <= 3;
}

int prefill_emulated_exp_columns(int tile_config) {
  if (tile_config < 0 || tile_config >= kPrefillNumTileConfigs) return -1;
  return kVariants[tile_config][0];
}

cudaError_t launch_prefill_sm100(const PrefillKernelArgs& args, const CUtensorMap& tm_q,
                                 const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                 int q_slots, int tile_config, int max_seqlen_q,
                                 cudaStream_t stream) {
  const int head_slots = args.pair_heads ? args.n_heads / 2 : args.n_heads;
  dim3 grid = args.q_fastest ? dim3(q_slots, head_slots, args.batch)
                             : dim3(head_slots, args.batch, q_slots);
  if (tile_config < 0 || tile_config >= kPrefillNumTileConfigs) return cudaErrorInvalidValue;
  int emu = kVariants[tile_config][0], h2 = kVariants[tile_config][1];
  if (tile_config == 0) {
    // Measured on B200 (interleaved A/B, GQA 32/8, R = 128): with interior tiles taking their
    // exponentials against the running max (no row-max pass), 2 FMA-pipe exponentials of 16
    // beat all-SFU by 0.5 % (32k causal), 3.6 % (window 4096) and 1.6 % (ragged), and 4 of 16
    // lose 4 % at 32k.
    emu = 2;
    h2 = 0;
  }
  if (args.kv_splits > 1) {  // KV split: the automatic choice, contiguous or paged K/V
    if (args.n_out_peers > 0 || emu != 2 || h2 != 0) return cudaErrorInvalidValue;
    grid = args.q_fastest ? dim3(q_slots * args.kv_splits, head_slots, args.batch)
                          : dim3(head_slots, args.batch, q_slots * args.kv_splits);
    if (args.block_table != nullptr)
      return launch_variant<2, 0, true, false, true>(args, tm_q, tm_k, tm_v, grid, stream);
    return launch_variant<2, 0, false, false, true>(args, tm_q, tm_k, tm_v, grid, stream);
  }
  if (args.n_out_peers > 0) {  // output copies on other GPUs: contiguous K/V, automatic choice
    if (args.block_table != nullptr || emu != 2 || h2 != 0) return cudaErrorInvalidValue;
    return launch_variant<2, 0, false, true>(args, tm_q, tm_k, tm_v, grid, stream);
  }
  if (args.block_table != nullptr) {  // paged cache: the automatic choice and its neighbours
    if (emu == 0 && h2 == 0) return launch_variant<0, 0, true>(args, tm_q, tm_k, tm_v, grid, stream);
    if (emu == 2 && h2 == 0) return launch_variant<2, 0, true>(args, tm_q, tm_k, tm_v, grid, stream);
    if (emu == 4 && h2 == 0) return launch_variant<4, 0, true>(args, tm_q, tm_k, tm_v, grid, stream);
    return cudaErrorInvalidValue;
  }
#define IFA4_VARIANT(E, H) \
  if (emu == E && h2 == H) return launch_variant<E, H, false>(args, tm_q, tm_k, tm_v, grid, stream);
  IFA4_VARIANT(0, 0)
  IFA4_VARIANT(2, 0)
  IFA4_VARIANT(4, 0)
  IFA4_VARIANT(6, 0)
  IFA4_VARIANT(8, 0)
  IFA4_VARIANT(0, 16)
  IFA4_VARIANT(0, 8)
  IFA4_VARIANT(4, 8)
#undef IFA4_VARIANT
  return cudaErrorInvalidValue;
}

}  // namespace ifa4
