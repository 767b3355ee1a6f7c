// W4A8 GEMM (packed int4 weights x int8 activations -> int32 in TMEM, fused
// epilogue) on tcgen05, with three decoupled shared-memory rings:
//
//   A ring       activations, TMA -> MMA                   (full_a / empty_a)
//   packed ring  int4_pack weight bytes, TMA -> unpack      (full_p / empty_p)
//   B ring       expanded int8 weights, unpack -> MMA       (ready_b / empty_b)
//
// The packed ring is deep (its stages are small), so weight bytes are
// prefetched far ahead; an unpack warp reads a packed chunk into registers,
// expands the nibbles there and writes the int8 row chunk into the B ring
// (128-byte swizzled, the layout the MMA's shared-memory descriptor reads).
// No stage is expanded in place, so unpack warps never wait for each other.
//
// kCta == 2 runs a CTA pair (cluster of two) on one 256 x 256 tile: each CTA
// holds 128 rows of A and 128 rows of B, the leader issues cta_group::2 MMAs
// and both CTAs' TMEM receive their 128 accumulator rows. Per SM this halves
// the weight bytes fetched, expanded and read by the tensor core.
//
// Warp roles: 0 A producer, 1 TMEM owner + MMA issuer, 2 packed producer,
// 4..11 epilogue (two sets of four, one per TMEM accumulator buffer), and
// eight unpack warps that avoid scheduler 1 (warp % 4 == 1), where the MMA
// warp issues: ALU-heavy warps on the issuing warp's scheduler slow
// tcgen05.mma issue several-fold.
#pragma once

#include "mma_kernel.cuh"

namespace w4a8 {

struct W4Roles {
  static constexpr int kEpiWarps = 8;
  static constexpr int kUnpackWarps = 8;
  static constexpr int kGroupWarps = 4;  // unpack warps per k-block (two groups alternate k-blocks)
  // Unpack warp u: warp 3, then warps 12.. whose index is not 1 mod 4.
  static constexpr __host__ __device__ int unpack_warp(int u) {
    if (u == 0) return 3;
    int n = 1;
    for (int w = 4 + kEpiWarps;; ++w) {
      if (w % 4 == 1) continue;
      if (n == u) return w;
      ++n;
    }
  }
  static constexpr __host__ __device__ int unpack_index(int warp) {
    for (int u = 0; u < kUnpackWarps; ++u)
      if (unpack_warp(u) == warp) return u;
    return -1;
  }
};
constexpr int kW4Threads = (W4Roles::unpack_warp(W4Roles::kUnpackWarps - 1) + 1) * 32;

constexpr int kMaxPkStages = 12;
constexpr int kMaxB8Stages = 8;

// Bounded waits on up to three barriers by lane 0; the warp gets the result.
__device__ __forceinline__ bool warp_wait_all(int lane, volatile int* abort_flag, uint64_t* b0, uint32_t p0,
                                              uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2) {
  int ok = 1;
  if (lane == 0)
    ok = (mbar_wait(b0, p0, abort_flag) && mbar_wait(b1, p1, abort_flag) && mbar_wait(b2, p2, abort_flag)) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Position in a ring of `n` stages: stage index and phase parity, advanced
// by `step` (< n + 1) per k-block without division.
struct RingPos {
  uint32_t s = 0, ph = 0;
  __device__ __forceinline__ void advance(uint32_t step, uint32_t n) {
    s += step;
    if (s >= n) { s -= n; ph ^= 1; }
  }
};

// Work unit u of the persistent loop: output tile (mt, nt) and the k-block
// range [kb0, kb1) of its split (one split covers all k-blocks).
struct Unit {
  int mt, nt, kb0, kb1;
};
__device__ __forceinline__ Unit unit_of(const KParams& p, int u) {
  Unit r;
  const int ks = u % p.k_splits;
  const int tile = u / p.k_splits;
  r.mt = tile / p.tiles_n;
  r.nt = tile - r.mt * p.tiles_n;
  r.kb0 = ks * p.kb_per_split;
  r.kb1 = min(r.kb0 + p.kb_per_split, p.num_kb);
  return r;
}

// Wait until the last fill of every stage of a ring has landed (no TMA may
// still be writing shared memory when the CTA exits). `q` fills were issued.
__device__ __forceinline__ void drain_ring(uint64_t* full, int stages, uint32_t q, volatile int* abort_flag) {
  for (int i = 0; i < stages && uint32_t(i) < q; ++i) {
    const uint32_t last = q - 1 - uint32_t(i);
    const unsigned long long t0 = global_timer_ns();
    while (!mbar_try_wait(&full[last % uint32_t(stages)], (last / uint32_t(stages)) & 1))
      if (global_timer_ns() - t0 > kWaitLimitNs) { *abort_flag = 1; break; }
  }
}

// kSwap (small M, split-K only): the MMA computes C^T = W . X^T, so the 128
// weight rows of a tile (output channels) are the MMA's M and TMEM lanes and
// BN tokens are its N. A warp then holds 32 consecutive channels of each
// token, and its split-K partial sums go out as 128-byte coalesced adds.
template <int BN, int kCta, bool kSwap>
__global__ void __launch_bounds__(kW4Threads, 1)
    w4a8_gemm_w4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ KParams p) {
  constexpr bool kPair = kCta == 2;
  static_assert(kCta == 1 || (kPair && BN == 256 && !kSwap), "CTA pairs use 256-wide tiles");
  constexpr int kBNL = kSwap ? kBM : BN / kCta;  // weight rows held by this CTA
  constexpr int kXRows = kSwap ? BN : kBM;       // activation rows per stage
  constexpr int kNB = 2;                        // TMEM accumulator buffers
  constexpr int kSetWarps = W4Roles::kEpiWarps / kNB;
  static_assert(kSetWarps == 4, "one epilogue warp per TMEM lane quadrant and buffer");
  constexpr uint32_t kTmemCols = uint32_t(kNB * BN) < 32u ? 32u : uint32_t(kNB * BN);
  constexpr int kGT = W4Roles::kGroupWarps * 32;  // unpack threads per k-block
  constexpr int kPer = kBNL * 8 / kGT;            // 16-byte int8 chunks per unpack thread and k-block
  static_assert(kPer >= 1 && kGT % 64 == 0, "unpack shape");
  constexpr uint32_t kPkBytes = kBNL * (kBK / 2);  // packed stage
  constexpr uint32_t kB8Bytes = kBNL * kBK;        // int8 stage

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_a[kMaxStages], empty_a[kMaxStages];
  __shared__ __align__(8) uint64_t full_p[kMaxPkStages], empty_p[kMaxPkStages];
  __shared__ __align__(8) uint64_t ready_b[kMaxB8Stages], empty_b[kMaxB8Stages];
  __shared__ __align__(8) uint64_t bar_tfull[kNB], bar_tempty[kNB], bar_drain;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const int tile0 = kPair ? int(blockIdx.x >> 1) : int(blockIdx.x);
  const int tstep = kPair ? int(gridDim.x >> 1) : int(gridDim.x);
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - smem_u32(smem_raw));
  const uint32_t Sa = uint32_t(p.stages), Sp = uint32_t(p.pk_stages), Sb = uint32_t(p.b8_stages);

  pdl_trigger();  // the next kernel of the stream may launch; it waits for this one in its own pdl_wait
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < Sa; ++s) { mbar_init(&full_a[s], 1); mbar_init(&empty_a[s], 1); }
    for (uint32_t s = 0; s < Sp; ++s) { mbar_init(&full_p[s], 1); mbar_init(&empty_p[s], W4Roles::kGroupWarps); }
    for (uint32_t s = 0; s < Sb; ++s) {
      mbar_init(&ready_b[s], kCta * W4Roles::kGroupWarps);
      mbar_init(&empty_b[s], 1);
    }
    for (int b = 0; b < kNB; ++b) {
      mbar_init(&bar_tfull[b], 1);
      mbar_init(&bar_tempty[b], kCta * kSetWarps);
    }
    mbar_init(&bar_drain, 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(&tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync();  // the peer's barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  pdl_wait();  // global memory only after the previous kernel of the stream has completed
  const int total_tiles = p.tiles_m * p.tiles_n * p.k_splits;  // work units

  if (warp == 0 || warp == 2) {
    // ------------------------- A / packed producers -------------------------
    if (lane == 0) {
      const bool is_a = warp == 0;
      uint64_t* full = is_a ? full_a : full_p;
      uint64_t* empty = is_a ? empty_a : empty_p;
      const uint32_t S = is_a ? Sa : Sp;
      uint8_t* ring = base + (is_a ? p.a_off : p.bp_off);
      const uint32_t stage_bytes = is_a ? uint32_t(kXRows * kBK) : kPkBytes;
      uint32_t q = 0;
      RingPos r;
      bool ok = true;
      for (int t = tile0; ok && t < total_tiles; t += tstep) {
        const Unit un = unit_of(p, t);
        const int row = is_a ? (kPair ? 2 * un.mt + int(rank) : un.mt) * kXRows : un.nt * (kSwap ? kBM : BN) + int(rank) * kBNL;
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++q, r.advance(1, S)) {
          if (!mbar_wait(&empty[r.s], r.ph ^ 1, &abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[r.s], stage_bytes);
          tma_load_2d(ring + r.s * stage_bytes, is_a ? &tmA : &tmW, &full[r.s], is_a ? kb * kBK : kb * (kBK / 2),
                      row);
        }
      }
      drain_ring(full, int(S), q, &abort_flag);
      if (!ok) atomicOr(p.err, kErrTimeoutProducer);
    }
  } else if (warp == 1) {
    // ------------------------------- MMA ------------------------------------
    if (lane == 0 && rank == 0) {  // in a CTA pair the leader issues for both
      constexpr uint32_t idesc = make_idesc_i8(kCta * kBM, BN);  // swap: M = 128 channels, N = BN tokens
      const uint64_t tmpl = make_smem_desc(0, 16, 1024, kLayoutSw128);
      const uint32_t a0 = (base_u32 + p.a_off) >> 4, b0 = (base_u32 + p.b_off) >> 4;
      constexpr uint32_t a_step = (kXRows * kBK) >> 4, b_step = kB8Bytes >> 4;
      RingPos ra, rb;
      int it = 0;
      bool ok = true;
      for (int t = tile0; ok && t < total_tiles; t += tstep, ++it) {
        const int buf = it & 1;
        if (!mbar_wait(&bar_tempty[buf], ((it >> 1) & 1) ^ 1, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        // No exits inside: a failed wait clears `ok` (later waits give up
        // within a few hundred polls) and the tile loop stops.
        const Unit un = unit_of(p, t);
        for (int kb = un.kb0; kb < un.kb1; ++kb, ra.advance(1, Sa), rb.advance(1, Sb)) {
          const uint32_t sa = ra.s, sb = rb.s;
          // ready_b: this k-block's weights are expanded and its A landed, in both CTAs of a pair.
          ok &= mbar_wait(&ready_b[sb], rb.ph, &abort_flag);
          tc_fence_after();
          const uint64_t xd = tmpl + (a0 + sa * a_step), wd = tmpl + (b0 + sb * b_step);
          const uint64_t ad = kSwap ? wd : xd, bd = kSwap ? xd : wd;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (kPair)
              mma_i8_ss_pair(d_tmem, ad + 2 * j, bd + 2 * j, idesc, ((kb - un.kb0) | j) != 0 ? 1u : 0u);
            else
              mma_i8_ss(d_tmem, ad + 2 * j, bd + 2 * j, idesc, ((kb - un.kb0) | j) != 0 ? 1u : 0u);
          }
          if constexpr (kPair) {
            mma_commit_pair_both(&empty_a[sa]);
            mma_commit_pair_both(&empty_b[sb]);
          } else {
            mma_commit(&empty_a[sa]);
            mma_commit(&empty_b[sb]);
          }
        }
        if (!ok) break;
        if constexpr (kPair)
          mma_commit_pair_both(&bar_tfull[buf]);
        else
          mma_commit(&bar_tfull[buf]);
      }
      if constexpr (kPair)
        mma_commit_pair_local(&bar_drain);
      else
        mma_commit(&bar_drain);
      const unsigned long long t0 = global_timer_ns();
      while (!mbar_try_wait(&bar_drain, 0))
        if (global_timer_ns() - t0 > kWaitLimitNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      if (!ok) atomicOr(p.err, kErrTimeoutMma);
    }
  } else if (warp >= 4 && warp < 4 + W4Roles::kEpiWarps) {
    // ----------------------------- epilogue --------------------------------
    const int q4 = warp & 3;                      // TMEM lane quadrant of this warp
    const int set = (warp - 4) / kSetWarps;        // accumulator buffer drained by this warp
    const int m = q4 * 32 + lane;
    EpiConsts k;
    k.rs = p.epi.out_kind == 3 ? __frcp_rn(p.epi.out_scale) : 1.0f;
    k.qnf = float(p.epi.qn);
    k.qpf = float(p.epi.qp);
    k.relu_in_clamp = p.epi.out_kind == 3 && p.epi.qn >= 0 && p.epi.aux == nullptr;
    int it = set;
    for (int t = tile0 + set * tstep; t < total_tiles; t += kNB * tstep, it += kNB) {
      int ok = 1;
      if (lane == 0) ok = mbar_wait_idle(&bar_tfull[set], (it >> 1) & 1, &abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicOr(p.err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const Unit un = unit_of(p, t);
      long long out_off = 0, prow = 0;
      const bool valid = !kSwap && row_coords<false>(p, kPair ? 2 * un.mt + int(rank) : un.mt, m, out_off, prow);
      const uint32_t t_addr = tmem_base + (uint32_t(q4 * 32) << 16) + set * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t acc[16];
        tmem_ld16(t_addr + c0, acc);
        tmem_ld_wait();
        if constexpr (kSwap) {
          // Lane = channel, columns = tokens: C[token][channel] += acc.
          const int ch = un.nt * kBM + m, tok0 = un.mt * BN + c0;
          if (ch < p.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (tok0 + i < p.M) atomicAdd(p.ws + (long long)(tok0 + i) * p.ws_ld + ch, int(acc[i]));
          }
        } else if (valid) {
          const int n = un.nt * BN + c0;
          if (p.k_splits > 1) {
            // Split-K: add this k-range's partial sums (int32 addition is
            // exact in any order); the finish kernel applies the epilogue.
            int* dst = p.ws + prow * p.ws_ld + n;
            const int nc = min(16, p.N - n);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (i < nc) atomicAdd(dst + i, int(acc[i]));
          } else {
            epilogue16(p.epi, k, acc, n, out_off + (long long)n * p.epi.s_ch, prow);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair)
          mbar_arrive_cluster(&bar_tempty[set], 0);  // the leader reuses the buffer once both CTAs drained it
        else
          mbar_arrive(&bar_tempty[set]);
      }
    }
  } else if (W4Roles::unpack_index(warp) >= 0) {
    // ------------------------------ unpack ---------------------------------
    // Group g (four warps) takes the k-blocks q with q % 2 == g. Thread gt
    // owns 16-byte int8 chunks gt + kGT * j of the stage: chunk (gt & 7) of
    // row (gt >> 3) + 16 j, whose swizzle term (row & 7) is the same for all j.
    const int u = W4Roles::unpack_index(warp);
    const uint32_t g = uint32_t(u / W4Roles::kGroupWarps);
    const int gt = (u % W4Roles::kGroupWarps) * 32 + lane;
    const uint32_t src0 = uint32_t(gt) * 8;
    const uint32_t dst0 = uint32_t(gt >> 3) * 128 + (uint32_t((gt & 7) ^ ((gt >> 3) & 7)) << 4);
    // This group's k-blocks are q = g, g + 2, ... of the CTA's sequence; the
    // ring positions advance with every k-block.
    RingPos ra, rp, rb;
    uint32_t q = 0;
    bool ok = true;
    for (int t = tile0; ok && t < total_tiles; t += tstep) {
      const Unit un = unit_of(p, t);
      for (int kb = un.kb0; kb < un.kb1; ++kb, ++q, ra.advance(1, Sa), rp.advance(1, Sp), rb.advance(1, Sb)) {
        if ((q & 1) != g) continue;
        const uint32_t sa = ra.s, sp = rp.s, sb = rb.s;
        if (!warp_wait_all(lane, &abort_flag, &full_p[sp], rp.ph, &empty_b[sb], rb.ph ^ 1, &full_a[sa], ra.ph)) {
          ok = false;
          break;
        }
        const uint8_t* pk = base + p.bp_off + sp * kPkBytes;
        uint8_t* b8 = base + p.b_off + sb * kB8Bytes;
        uint2 v[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) v[j] = *reinterpret_cast<const uint2*>(pk + src0 + j * kGT * 8);
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          uint4 o;
          unpack_nibbles8(v[j].x, o.x, o.y);
          unpack_nibbles8(v[j].y, o.z, o.w);
          *reinterpret_cast<uint4*>(b8 + dst0 + j * kGT * 16) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty_p[sp]);  // the packed bytes were consumed above
          if constexpr (kPair)
            mbar_arrive_cluster(&ready_b[sb], 0);
          else
            mbar_arrive(&ready_b[sb]);
        }
      }
    }
    if (!ok && lane == 0) atomicOr(p.err, kErrTimeoutUnpack);
  }

  tc_fence_before();
  __syncthreads();
  // A pair leaves together: no remote arrive or operand read may reach an
  // exited CTA, and both CTAs free their TMEM at once.
  if constexpr (kPair) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Split-K finish: the fused epilogue over the int32 sums; one thread per
// (row, 16 columns).
__global__ void __launch_bounds__(256) w4a8_splitk_finish_kernel(const __grid_constant__ KParams p) {
  pdl_trigger();
  pdl_wait();
  const int chunks = (p.N + 15) / 16;
  const long long idx = blockIdx.x * 256LL + threadIdx.x;
  if (idx >= (long long)p.M * chunks) return;
  const int row = int(idx / chunks);
  const int n = int(idx - (long long)row * chunks) * 16;
  EpiConsts k;
  k.rs = p.epi.out_kind == 3 ? __frcp_rn(p.epi.out_scale) : 1.0f;
  k.qnf = float(p.epi.qn);
  k.qpf = float(p.epi.qp);
  k.relu_in_clamp = p.epi.out_kind == 3 && p.epi.qn >= 0 && p.epi.aux == nullptr;
  const int* src = p.ws + row * p.ws_ld + n;
  uint32_t acc[16];
  if (n + 16 <= p.N && (p.ws_ld & 3) == 0) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int4 v = *reinterpret_cast<const int4*>(src + 4 * g);
      acc[4 * g] = uint32_t(v.x);
      acc[4 * g + 1] = uint32_t(v.y);
      acc[4 * g + 2] = uint32_t(v.z);
      acc[4 * g + 3] = uint32_t(v.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = n + i < p.N ? uint32_t(src[i]) : 0u;
  }
  epilogue16(p.epi, k, acc, n, (long long)row * p.epi.s_pix + (long long)n * p.epi.s_ch, row);
}

}  // namespace w4a8
