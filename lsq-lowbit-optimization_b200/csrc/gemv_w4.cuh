// W4A8 GEMV for a few tokens (M <= 8): C[M, N] = epilogue(X[M, K] . W[N, K]^T)
// on the CUDA cores, streaming the packed weights straight from HBM into
// registers (no shared-memory staging: at these shapes the weight bytes are
// the whole cost, and staging them through shared memory for the tensor
// cores caps the stream well below HBM bandwidth).
//
// Nibble arithmetic: an int4_pack byte holds element 2j in its low and 2j+1
// in its high nibble (two's complement). For a nibble n, w' = n ^ 8 lies in
// [0, 15] and the weight is w' - 8, so
//   sum_k w_k x_k = sum_k w'_k x_k - 8 * sum_k x_k,
// with w' obtained by one mask-and-xor per 4 nibbles and the products on
// dp4a against the activations de-interleaved into even / odd elements.
// All of it is exact int32 arithmetic.
//
// Lane-per-row form (3..8 tokens): block = 32 output channels (one per lane) x
// kGemvWarps warps, each warp a contiguous K range; the warps' partial sums
// are added in shared memory and the fused epilogue (epilogue16) runs on
// 16-channel chunks per token. More tokens (small GEMMs whose tensor-core
// tiles could not fill the GPU) run as a second grid dimension of 8-token
// groups: block (x, y) takes channels 32 x .. and tokens 8 y ... The
// row-per-warp form below serves 1-2 tokens.
#pragma once

#include "mma_kernel.cuh"

namespace w4a8 {

constexpr int kGemvWarps = 16;
constexpr int kGemvMaxTokens = 8;
constexpr int kGemvUnroll2 = 2;  // lane-per-row form: 32-byte weight chunks in flight per lane
constexpr int kGemvRows = kGemvWarps;  // row-per-warp form: output channels per block
constexpr int kGemvUnroll = 8;         // row-per-warp form: 16-byte chunks in flight per lane

__device__ __forceinline__ int dp4a_s8(uint32_t a, uint32_t b, int c) {
  return __dp4a(int(a), int(b), c);
}

// smem: xs[MT][K / 4] words (per group of 8 elements: even word, odd word),
// red[kGemvWarps][MT][32] int32, fin[MT][32] int32, xsum[MT].
template <int MT>
__global__ void __launch_bounds__(kGemvWarps * 32) w4a8_gemv_w4_kernel(const int8_t* __restrict__ X, long long ldx,
                                                                       const uint8_t* __restrict__ W, long long ldw,
                                                                       int M, int N, int K,
                                                                       const __grid_constant__ EpiParams e) {
  extern __shared__ __align__(16) uint32_t gsm[];
  pdl_trigger();
  pdl_wait();
  const int t0 = int(blockIdx.y) * MT;  // this block's first token
  X += (long long)t0 * ldx;
  M = min(M - t0, MT);
  const int kw = K / 4;  // de-interleaved words per token
  uint32_t* xs = gsm;
  int* red = reinterpret_cast<int*>(xs + MT * kw);
  int* fin = red + kGemvWarps * MT * 32;
  int* xsum = fin + MT * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid < MT) xsum[tid] = 0;
  __syncthreads();
  // X rows -> even / odd words (16 bytes = two groups of 8 elements per step).
  for (int t = 0; t < MT; ++t) {
    int sx = 0;
    for (int i = tid; i < K / 16; i += kGemvWarps * 32) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t < M) v = *reinterpret_cast<const uint4*>(X + t * ldx + i * 16);
      sx = dp4a_s8(v.x, 0x01010101u, sx);
      sx = dp4a_s8(v.y, 0x01010101u, sx);
      sx = dp4a_s8(v.z, 0x01010101u, sx);
      sx = dp4a_s8(v.w, 0x01010101u, sx);
      uint4 o;
      o.x = __byte_perm(v.x, v.y, 0x6420);  // elements 0 2 4 6
      o.y = __byte_perm(v.x, v.y, 0x7531);  // elements 1 3 5 7
      o.z = __byte_perm(v.z, v.w, 0x6420);
      o.w = __byte_perm(v.z, v.w, 0x7531);
      *reinterpret_cast<uint4*>(xs + t * kw + i * 4) = o;
    }
#pragma unroll
    for (int d = 16; d; d >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, d);
    if (lane == 0 && sx) atomicAdd(&xsum[t], sx);
  }
  __syncthreads();

  // This warp's K range, in 64-element (32-byte) chunks.
  const int chunks = K / 64;
  const int per = (chunks + kGemvWarps - 1) / kGemvWarps;
  const int c0 = warp * per, c1 = min(c0 + per, chunks);
  const int n = blockIdx.x * 32 + lane;
  int acc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) acc[t] = 0;
  if (n < N) {
    const uint8_t* wrow = W + (long long)n * ldw;
#pragma unroll(kGemvUnroll2)
    for (int c = c0; c < c1; ++c) {
      const uint4 wa = __ldg(reinterpret_cast<const uint4*>(wrow + c * 32));
      const uint4 wb = __ldg(reinterpret_cast<const uint4*>(wrow + c * 32 + 16));
      const uint32_t words[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t lo = (words[i] & 0x0F0F0F0Fu) ^ 0x08080808u;          // w' of elements 0 2 4 6
        const uint32_t hi = ((words[i] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;   // w' of elements 1 3 5 7
        const int g = c * 8 + i;                                              // group of 8 elements
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const uint2 xv = *reinterpret_cast<const uint2*>(xs + t * kw + 2 * g);
          acc[t] = dp4a_s8(lo, xv.x, acc[t]);
          acc[t] = dp4a_s8(hi, xv.y, acc[t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) red[(warp * MT + t) * 32 + lane] = acc[t];
  __syncthreads();
  if (tid < MT * 32) {
    const int t = tid / 32, l = tid % 32;
    int s = 0;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) s += red[(w * MT + t) * 32 + l];
    fin[t * 32 + l] = s - 8 * xsum[t];
  }
  __syncthreads();
  if (tid < MT * 2) {
    const int t = tid / 2, h = tid % 2;
    if (t < M) {
      EpiConsts k;
      k.rs = e.out_kind == 3 ? __frcp_rn(e.out_scale) : 1.0f;
      k.qnf = float(e.qn);
      k.qpf = float(e.qp);
      k.relu_in_clamp = e.out_kind == 3 && e.qn >= 0 && e.aux == nullptr;
      uint32_t a16[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) a16[i] = uint32_t(fin[t * 32 + h * 16 + i]);
      const int nc = blockIdx.x * 32 + h * 16;
      epilogue16(e, k, a16, nc, (long long)(t0 + t) * e.s_pix + (long long)nc * e.s_ch, t0 + t);
    }
  }
}

// Row-per-warp form for one or two tokens: each warp owns a weight row and its
// lanes read consecutive 16-byte chunks (512 coalesced bytes per load,
// kGemvUnroll loads in flight per lane); a warp shuffle adds the lanes. With
// more tokens the per-lane activation reads from shared memory dominate and
// the lane-per-row form above is faster.
// smem: xs[MT][K / 4] words, fin[MT][kGemvRows] int32, xsum[MT].
template <int MT>
__global__ void __launch_bounds__(kGemvWarps * 32) w4a8_gemv_w4_rows_kernel(const int8_t* __restrict__ X, long long ldx,
                                                                       const uint8_t* __restrict__ W, long long ldw,
                                                                       int M, int N, int K,
                                                                       const __grid_constant__ EpiParams e) {
  extern __shared__ __align__(16) uint32_t gsm[];
  pdl_trigger();
  pdl_wait();
  const int kw = K / 4;  // de-interleaved words per token
  uint32_t* xs = gsm;
  int* fin = reinterpret_cast<int*>(xs + MT * kw);
  int* xsum = fin + MT * kGemvRows;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid < MT) xsum[tid] = 0;
  __syncthreads();
  // X rows -> even / odd words (16 bytes = two groups of 8 elements per step).
  for (int t = 0; t < MT; ++t) {
    int sx = 0;
    for (int i = tid; i < K / 16; i += kGemvWarps * 32) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t < M) v = *reinterpret_cast<const uint4*>(X + t * ldx + i * 16);
      sx = dp4a_s8(v.x, 0x01010101u, sx);
      sx = dp4a_s8(v.y, 0x01010101u, sx);
      sx = dp4a_s8(v.z, 0x01010101u, sx);
      sx = dp4a_s8(v.w, 0x01010101u, sx);
      uint4 o;
      o.x = __byte_perm(v.x, v.y, 0x6420);  // elements 0 2 4 6
      o.y = __byte_perm(v.x, v.y, 0x7531);  // elements 1 3 5 7
      o.z = __byte_perm(v.z, v.w, 0x6420);
      o.w = __byte_perm(v.z, v.w, 0x7531);
      *reinterpret_cast<uint4*>(xs + t * kw + i * 4) = o;
    }
#pragma unroll
    for (int d = 16; d; d >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, d);
    if (lane == 0 && sx) atomicAdd(&xsum[t], sx);
  }
  __syncthreads();

  // Row n of this warp: lane l reads bytes [16 (l + 32 i), +16) of it, i.e.
  // K elements [32 (l + 32 i), +32) = four groups of 8 (x words 8 (l + 32 i) ..).
  const int n = blockIdx.x * kGemvRows + warp;
  int acc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) acc[t] = 0;
  if (n < N) {
    const uint8_t* wrow = W + (long long)n * ldw;
    const int nchunk = K / 32;  // 16-byte chunks in the row
    for (int c0 = 0; c0 < nchunk; c0 += 32 * kGemvUnroll) {
      uint4 wv[kGemvUnroll];
#pragma unroll
      for (int u = 0; u < kGemvUnroll; ++u) {
        const int c = c0 + 32 * u + lane;
        wv[u] = c < nchunk ? __ldg(reinterpret_cast<const uint4*>(wrow + c * 16))
                           : make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // w' = 0
      }
#pragma unroll
      for (int u = 0; u < kGemvUnroll; ++u) {
        const int c = min(c0 + 32 * u + lane, nchunk - 1);  // padding chunks (w' = 0) read a valid x slice
        const uint32_t words[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const uint4 xa = *reinterpret_cast<const uint4*>(xs + t * kw + 8 * c);
          const uint4 xb = *reinterpret_cast<const uint4*>(xs + t * kw + 8 * c + 4);
          const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t lo = (words[i] & 0x0F0F0F0Fu) ^ 0x08080808u;         // w' of elements 0 2 4 6
            const uint32_t hi = ((words[i] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;  // w' of elements 1 3 5 7
            acc[t] = dp4a_s8(lo, xw[2 * i], acc[t]);
            acc[t] = dp4a_s8(hi, xw[2 * i + 1], acc[t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    int v = acc[t];
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    if (lane == 0) fin[t * kGemvRows + warp] = v - 8 * xsum[t];
  }
  __syncthreads();
  constexpr int kHalves = kGemvRows / 16;
  if (tid < MT * kHalves) {
    const int t = tid / kHalves, h = tid % kHalves;
    if (t < M) {
      EpiConsts k;
      k.rs = e.out_kind == 3 ? __frcp_rn(e.out_scale) : 1.0f;
      k.qnf = float(e.qn);
      k.qpf = float(e.qp);
      k.relu_in_clamp = e.out_kind == 3 && e.qn >= 0 && e.aux == nullptr;
      uint32_t a16[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) a16[i] = uint32_t(fin[t * kGemvRows + h * 16 + i]);
      const int nc = blockIdx.x * kGemvRows + h * 16;
      epilogue16(e, k, a16, nc, (long long)t * e.s_pix + (long long)nc * e.s_ch, t);
    }
  }
}

inline size_t gemv_rows_smem_bytes(int mt, int K) {
  return size_t(mt) * size_t(K) + size_t(mt) * kGemvRows * 4 + size_t(mt) * 4;
}

inline size_t gemv_smem_bytes(int mt, int K) {
  return size_t(mt) * size_t(K) + size_t(kGemvWarps) * mt * 32 * 4 + size_t(mt) * 32 * 4 + size_t(mt) * 4;
}

}  // namespace w4a8
