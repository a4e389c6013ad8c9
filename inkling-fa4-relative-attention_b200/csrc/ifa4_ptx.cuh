// Inline-PTX building blocks for sm_100a: mbarriers with bounded waits, TMA tensor loads
// (no multicast), tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads/stores) and the
// shared-memory matrix descriptors UMMA consumes.
//
// Descriptor formats (bit positions) follow the public sm_100 UMMA definitions as written in
// CUTLASS's cute/arch/mma_sm100_desc.hpp (SmemDescriptor, InstrDescriptor).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ifa4 {

// Bound on any spin-wait inside a kernel.  A legitimate wait lasts microseconds; if one ever
// exceeds this the kernel records IFA4 status bits, raises the CTA/grid abort flags and
// unwinds instead of hanging the GPU.
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ---------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Abort state shared by all waits of one CTA: a shared-memory flag (this CTA) and a global
// status word (all CTAs of all launches until cleared by the host).
struct AbortCtx {
  volatile int* cta_flag;  // shared memory
  int* status;             // global memory (may be null)
  int status_bit;
};

__device__ __forceinline__ bool abort_requested(const AbortCtx& a) {
  if (*a.cta_flag) return true;
  if (a.status != nullptr && *reinterpret_cast<volatile int*>(a.status) != 0) return true;
  return false;
}

__device__ __forceinline__ void raise_abort(const AbortCtx& a) {
  *a.cta_flag = 1;
  if (a.status != nullptr) atomicOr(a.status, a.status_bit);
  __threadfence();
}

// Single-thread bounded wait.  Returns false if the wait was abandoned (timeout or abort).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const AbortCtx& a,
                                          unsigned long long timeout_ns = kWaitTimeoutNs) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 255u) == 0) {
      if (abort_requested(a)) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        raise_abort(a);
        return false;
      }
    }
  }
}

// Warp-collective bounded wait: every lane polls, the outcome is warp-uniform.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, const AbortCtx& a,
                                               unsigned long long timeout_ns = kWaitTimeoutNs) {
  const uint32_t addr = smem_u32(bar);
  if (__all_sync(0xffffffffu, mbar_try_wait(addr, parity))) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (__all_sync(0xffffffffu, mbar_try_wait(addr, parity))) return true;
    if ((it & 255u) == 0) {
      int give_up = 0;
      if (lane_id() == 0) {
        if (abort_requested(a)) {
          give_up = 1;
        } else if (globaltimer_ns() - t0 > timeout_ns) {
          raise_abort(a);
          give_up = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
    }
  }
}

// ---------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), never with .multicast::cluster
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map,
                                                 uint64_t* bar, int c0, int c1, int c2,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_hint(void* smem_dst, const CUtensorMap* map,
                                                 uint64_t* bar, int c0, int c1, int c2, int c3,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads
// (TMA / tcgen05.mma operands) of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMA tensor store of a shared-memory box (bulk-group completion).  Coordinates must be
// non-negative; the part of the box beyond the tensor's extent is not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Returns once the shared-memory sources of every committed bulk store have been read.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Returns once every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 16-byte asynchronous global -> shared copy (L2 only; both addresses 16-byte aligned) and the
// wait for every such copy of this thread.
__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr), "l"(gptr)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// ---------------------------------------------------------------------------------------
// tcgen05: TMEM allocation
// ---------------------------------------------------------------------------------------
// Whole warp.  Writes the allocated TMEM base address to *smem_slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05: UMMA descriptors and issue
// ---------------------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100 version bits.
//   bits [0,14)  start address >> 4
//   bits [16,30) leading-dimension byte offset >> 4
//   bits [32,46) stride-dimension byte offset >> 4
//   bits [46,48) version = 1
//   bits [61,64) layout type (2 = SWIZZLE_128B)
// K-major, SW128: rows of 128 B, 8-row atoms 1024 B apart (SBO = 1024); LBO unused (1).
// MN-major, SW128: 64 contiguous MN elements per 128-B row; LBO = byte distance between
// successive 64-element MN blocks, SBO = distance between successive 8-row K groups.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Descriptor of the same matrix layout starting `off_bytes` further (off < 256 KB - start):
// the start address is the low 14-bit field in 16-byte units, so the add cannot carry out of
// it.  Volatile so the compiler re-derives it at each use instead of keeping every descriptor
// of an unrolled loop live in registers.
__device__ __forceinline__ uint64_t sdesc_advance(uint64_t desc, uint32_t off_bytes) {
  uint64_t r;
  asm volatile("add.u64 %0, %1, %2;" : "=l"(r) : "l"(desc), "l"(static_cast<uint64_t>(off_bytes >> 4)));
  return r;
}

// Instruction descriptor, kind::f16, bf16 x bf16 -> f32, dense.
//   [4,6) D format (1 = f32)  [7,10) A format (1 = bf16)  [10,13) B format (1 = bf16)
//   [15] A major (0 = K)  [16] B major (0 = K, 1 = MN)  [17,23) N >> 3  [24,29) M >> 4
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 op of this thread completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05: TMEM <-> registers (32 lanes x 32 bit, one TMEM lane per thread)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes (one register per column).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// Math helpers
// ---------------------------------------------------------------------------------------
// 2^x on the SFU (PTX ex2.approx.ftz.f32): ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (Blackwell f32x2 arithmetic): one instruction operates on two floats.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// max of three floats in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of floats on the FMA pipe instead of the SFU.
// Range reduction (Cody-Waite for base 2 needs no split constant): n = round(x) obtained by
// adding the rounding constant 1.5 * 2^23, f = x - n in [-1/2, 1/2]; 2^f by a degree-3
// polynomial minimising the relative error on [-1/2, 1/2] (Remez exchange; max relative error
// 7.5e-5, well under the 2^-9 half-ulp of the bf16 the result is rounded to); 2^n is applied by
// adding n to the exponent field (bits(t) << 23 == n << 23 modulo 2^32 for t = 1.5 * 2^23 + n).
// Inputs are clamped to >= -125 (the result is then ~2^-125 rather than 0) and must be <= 127.
__device__ __forceinline__ void exp2_poly_pair(float x0, float x1, float& y0, float& y1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -125.0f);
  x1 = fmaxf(x1, -125.0f);
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t r2 = f2_pack(kRound, kRound);
  const uint64_t t = f2_add(x, r2);
  const uint64_t f = f2_sub(x, f2_sub(t, r2));
  uint64_t p = f2_fma(f2_pack(0.0551716685f, 0.0551716685f), f,
                      f2_pack(0.2426111251f, 0.2426111251f));
  p = f2_fma(p, f, f2_pack(0.6932609677f, 0.6932609677f));
  p = f2_fma(p, f, f2_pack(0.9999280572f, 0.9999280572f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// exp2_poly_pair with the inputs also capped at 64 (result <= 2^64): for callers whose
// arguments may exceed 127, where the exponent insertion above would wrap; a capped result is
// still far above anything they accept, so the cap never changes an accepted value.
__device__ __forceinline__ void exp2_poly_pair_capped(float x0, float x1, float& y0, float& y1) {
  exp2_poly_pair(fminf(x0, 64.0f), fminf(x1, 64.0f), y0, y1);
}

// 2^x for a pair of floats with one SFU instruction (ex2.approx.f16x2): the inputs are rounded
// to fp16 (10-bit mantissa; the arguments are <= 8 here, so the input rounding changes the
// result by at most 0.14 %, below the bf16 rounding applied to it next) and the fp16 results
// are widened back.  Inputs below -25 give 0 or an fp16 subnormal (< 2^-24).
__device__ __forceinline__ void exp2_h2_pair(float x0, float x1, float& y0, float& y1) {
  uint32_t h, e;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(x1), "f"(x0));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(h));
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(y0), "=f"(y1)
      : "r"(e));
}

// ---------------------------------------------------------------------------------------
// Relative-bias windows (prefill and backward dQ)
// ---------------------------------------------------------------------------------------
// Vector bias path (rel 16-byte aligned, rel_extent a multiple of 8): chunk cc (columns
// [32 cc, 32 cc + 32)) of a tile whose column 0 sits at bias distance dtop needs this row's
// distances [dtop - 32 cc - 31, dtop - 32 cc].  The 40-element window from the 8-aligned
// distance below that range is loaded as five 16-byte vectors; a vector is either wholly inside
// [0, rel_extent) or wholly outside it (then zero, not read), so nothing outside the row's
// rel_extent elements is touched.
__device__ __forceinline__ void load_bias_window(const uint16_t* rel_row, int dtop, int cc,
                                                 int rel_extent, bool active, uint32_t (&w)[20]) {
  const int base = (dtop - 32 * cc - 31) & ~7;
#pragma unroll
  for (int v = 0; v < 5; ++v) {
    const int st = base + 8 * v;
    uint4 x = make_uint4(0u, 0u, 0u, 0u);
    if (active && st >= 0 && st < rel_extent) x = ldg_nc_v4(rel_row + st);
    w[4 * v] = x.x;
    w[4 * v + 1] = x.y;
    w[4 * v + 2] = x.z;
    w[4 * v + 3] = x.w;
  }
}

// b[i] = bias of column i of chunk cc, from the window above: column i has distance
// dtop - 32 cc - i = element (off + 31 - i) of the window, off = (dtop - 32 cc - 31) mod 8; the
// window is shifted by off elements with selects and a byte permute (no shared memory).
// Columns outside [0, rel_extent) read 0 from the zero-filled vectors.
__device__ __forceinline__ void bias_window_floats(const uint32_t (&w)[20], int dtop, int cc,
                                                   float (&b)[32]) {
  const int off = (dtop - 32 * cc - 31) & 7;
  const int q = off >> 1;  // whole words to skip
  uint32_t t2[17];
#pragma unroll
  for (int k = 0; k < 17; ++k)
    t2[k] = (q & 2) ? ((q & 1) ? w[k + 3] : w[k + 2]) : ((q & 1) ? w[k + 1] : w[k]);
  const uint32_t sel = (off & 1) ? 0x5432u : 0x3210u;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int j = 31 - i;  // element j of the shifted window
    const uint32_t pr = __byte_perm(t2[j >> 1], t2[(j >> 1) + 1], sel);
    b[i] = __uint_as_float((j & 1) ? (pr & 0xffff0000u) : (pr << 16));
  }
}

// x[i] += log2(e) * bias of column i of chunk cc.
__device__ __forceinline__ void add_bias_window(const uint32_t (&w)[20], int dtop, int cc,
                                                float (&x)[32]) {
  float b[32];
  bias_window_floats(w, dtop, cc, b);
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] += b[i] * 1.4426950408889634f;
}

// Warpgroup-wide register re-split (every warp of the warpgroup executes it; the sum over the
// CTA's warps must fit in the registers the CTA was launched with).
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegs) : "memory");
}
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegs) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x (low 16 bits) = lo
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

}  // namespace ifa4
