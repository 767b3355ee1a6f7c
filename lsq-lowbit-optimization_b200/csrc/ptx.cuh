// Blackwell (sm_100a) PTX building blocks used by every kernel of libw4a8:
// mbarriers with bounded waits, TMA tiled loads, tcgen05 TMEM allocation,
// int8 MMA issue/commit and TMEM loads, UMMA shared-memory descriptors.
//
// Everything here is written against the public PTX ISA (8.7) description of
// the tcgen05 / cp.async.bulk.tensor / mbarrier instructions.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "launch.cuh"

namespace w4a8 {

// ---------------------------------------------------------------------------
// Device error word. A kernel that gives up on a wait (a pipeline partner
// never arrived) records a code here and unwinds instead of hanging the GPU.
// ---------------------------------------------------------------------------
enum DeviceError : unsigned {
  kErrNone = 0,
  kErrTimeoutProducer = 1u << 0,
  kErrTimeoutMma = 1u << 1,
  kErrTimeoutEpilogue = 1u << 2,
  kErrTimeoutUnpack = 1u << 3,
  kErrTimeoutDrain = 1u << 4,
};

// ~2 s at any plausible clock: far above any legitimate wait in these kernels.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------- mbarrier ------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Spin part of mbar_wait, kept out of line: an inlined spin loop inside the
// MMA issue loop slows that loop down even when it is never entered.
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const unsigned long long t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Counterpart for long waits (an epilogue warp set waiting for its next
// accumulator tile): plain try_wait polls, with the abort flag and the time
// limit checked after every try. A try_wait with a suspend-time hint (20 us)
// used to sit here so that idle warps would take no issue slots; a trace of
// the 256 x 1000 x 512 GEMM showed the sleeping epilogue noticing its full
// accumulator about 3 us after the MMAs completed, and the polling form
// measured faster everywhere (layer-1 3x3 conv 89.8 -> 83.5 us).
__device__ __noinline__ bool mbar_wait_idle_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_idle_slow(bar, parity, abort_flag);
}

// Idle (abort flag checked every try) or spinning wait, chosen per kernel.
template <bool kIdle>
__device__ __forceinline__ bool mbar_wait_t(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  return kIdle ? mbar_wait_idle_slow(bar, parity, abort_flag) : mbar_wait_slow(bar, parity, abort_flag);
}

// Bounded wait for the phase with the given parity. Returns false (and sets
// *abort) when the limit passes or another role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, abort_flag);
}

// AND of `v` over the `count` threads meeting at named barrier `id`; every
// participant gets the same answer, so a group can abort uniformly.
__device__ __forceinline__ bool bar_and(uint32_t id, uint32_t count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------- TMA ---------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// ------------------------------ tcgen05 ------------------------------------
// TMEM allocation is warp-collective; the base address is written to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, issued by one thread.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// mma_i8_ss issued by one elected lane of a converged warp (every lane calls it).
__device__ __forceinline__ void mma_i8_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// mma_commit by one elected lane of a converged warp (every lane calls it).
__device__ __forceinline__ void mma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Arrive on an mbarrier once every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// ---- CTA pairs (cluster of 2, cta_group::2) --------------------------------
// A pair computes a 256-row tile: each CTA holds 128 rows of A and half of
// the tile's B rows, the pair's tensor cores exchange the B halves, and each
// CTA's TMEM receives its 128 accumulator rows. Only the leader (rank 0)
// issues MMAs; shared-memory operands sit at the same offsets in both CTAs.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on the mbarrier at this offset in CTA `rank` of the cluster (default
// release semantics; shared-memory writes meant for the tensor core are
// ordered before it by fence.proxy.async). A cluster-scope release here
// delays the arrival by thousands of cycles.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// Wait for a phase completed (partly) by the peer CTA. The peer arrives with
// release at cluster scope after making its shared-memory writes visible to
// the async proxy; polling stays at CTA scope (a cluster-scope acquire on
// every poll slows the SM's other shared-memory traffic), as for the
// tensor-core consumers of TMA data.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort_flag);
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[256 x N] (+)= A[256 x 32] * B[32 x N] over the pair; issued by the leader.
__device__ __forceinline__ void mma_i8_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at this offset in both CTAs of the pair once every
// tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(uint16_t(3))
      : "memory");
}
__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns: thread i of the warp receives
// lane (quadrant*32 + i), columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------- UMMA descriptors --------------------------------
// Shared-memory matrix descriptor (tcgen05 form): start>>4 [0,14), LBO>>4
// [16,30), SBO>>4 [32,46), version 1 at [46,48), base offset 0, layout type
// at [61,64): 0 = no swizzle (8x16B core matrices), 2 = 128B swizzle.
constexpr uint32_t kLayoutNone = 0;
constexpr uint32_t kLayoutSw128 = 2;
constexpr uint32_t kLayoutSw64 = 4;
constexpr uint32_t kLayoutSw32 = 6;

// base_offset [49,52) stays 0 here: the swizzle pattern is taken from the
// absolute shared-memory address bits, the same bits the TMA swizzled by.
// The start-address field holds addr >> 4 in 14 bits; every shared-memory
// address is below 2^18, so a template built for address 0 becomes the
// descriptor of address `a` by adding a >> 4 (no carry out of the field).
// Hot loops add to precomputed templates instead of re-encoding.
__host__ __device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                            uint32_t layout, uint32_t base_offset = 0) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(base_offset & 7u) << 49;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::i8: signed A and B, int32 D, K-major
// operands, M = 128, N = n.
__host__ __device__ constexpr uint32_t make_idesc_i8(uint32_t m, uint32_t n) {
  return (2u << 4)             // D format: S32
         | (1u << 7)           // A: signed 8-bit
         | (1u << 10)          // B: signed 8-bit
         | ((n >> 3) << 17)    // N >> 3
         | ((m >> 4) << 24);   // M >> 4
}

// ------------------------- int4 nibble unpack ------------------------------
// One 32-bit word holds 8 two's-complement nibbles; byte j carries element 2j
// in its low nibble and element 2j+1 in its high nibble. Produces the eight
// sign-extended int8 values in element order (two words).
__device__ __forceinline__ void unpack_nibbles8(uint32_t w, uint32_t& out_lo, uint32_t& out_hi) {
  // Per byte: t = nibble ^ 8 in [0,15]; (t + 0x78) ^ 0x80 == t - 8 as int8.
  const uint32_t lo = (w & 0x0F0F0F0Fu) ^ 0x08080808u;          // even elements
  const uint32_t hi = ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;   // odd elements
  const uint32_t slo = (lo + 0x78787878u) ^ 0x80808080u;
  const uint32_t shi = (hi + 0x78787878u) ^ 0x80808080u;
  out_lo = __byte_perm(slo, shi, 0x5140);  // e0 e1 e2 e3
  out_hi = __byte_perm(slo, shi, 0x7362);  // e4 e5 e6 e7
}

}  // namespace w4a8
