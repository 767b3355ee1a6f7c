// Persistent, warp-specialised tcgen05 int8 kernel shared by the W4A8 GEMM
// and the implicit-GEMM NHWC convolution.
//
//   D[128 x BN] (int32, TMEM) = A[128 x K] (int8, smem) . B[BN x K]^T (int8, smem)
//
// Rows of A are GEMM rows (GEMM mode) or a 16x8 block of output pixels of
// one image (conv mode); columns are output features / channels.
//
// Warp roles (Roles<conv>: 768 threads for the conv, 512 for the GEMM):
//   warp 0       TMA producer (one elected lane)
//   warp 1       TMEM owner + MMA issuer (one elected lane)
//   warps 4..    epilogue (16 or 8 warps): tcgen05.ld -> fused LSQ epilogue ->
//                global stores; warp w reads TMEM lanes 32*(w%4).. and the
//                column slice (w-4)/4 of the tile
//   last warps  int4 unpack (4 conv / 8 GEMM): the packed nibbles land (TMA) in the upper half
//                of the int8 B stage and are expanded in place into the
//                128B-swizzled int8 tile
// The accumulator is double-buffered in TMEM so the epilogue of tile i
// overlaps the main loop of tile i+1.
#pragma once

#include <cuda_fp16.h>

#include <climits>

#include "ptx.cuh"

namespace w4a8 {

constexpr int kBM = 128;          // rows per tile (MMA M)
constexpr int kBK = 128;          // K bytes per k-block (one 128B swizzle atom)
// Epilogue warps: the conv (short K, epilogue-heavy) uses 16, the GEMM
// (long K, main-loop bound) 8. The unpack warps follow them: 4 for the
// conv, 8 for the GEMM, whose weight expansion runs every k-block.
template <bool kConv>
struct Roles {
  static constexpr int kEpiWarps = kConv ? 16 : 8;
  static constexpr int kUnpackWarps = kConv ? 4 : 8;
  static constexpr int kUnpackWarp0 = 4 + kEpiWarps;
  static constexpr int kThreads = (kUnpackWarp0 + kUnpackWarps) * 32;
};

// TMEM accumulator buffers (tiles in flight between the MMA and the
// epilogue): as many as TMEM (512 columns) and the epilogue warp sets (one
// set of >= 4 warps per buffer) allow, at most 4. Each epilogue warp set
// drains one buffer, so short-K tiles overlap their epilogues.
__host__ __device__ constexpr int acc_buffers(int bn, bool conv) {
  const int by_warps = (conv ? Roles<true>::kEpiWarps : Roles<false>::kEpiWarps) / 4;
  const int by_tmem = 512 / bn;
  const int nb = by_warps < by_tmem ? by_warps : by_tmem;
  return nb < 4 ? nb : 4;
}
__host__ __device__ constexpr uint32_t tmem_columns(int bn, bool conv) {
  const uint32_t need = uint32_t(acc_buffers(bn, conv) * bn);
  uint32_t cols = 32;
  while (cols < need) cols <<= 1;
  return cols;
}
constexpr int kMaxStages = 8;
constexpr int kMaxHaloStages = 12;
constexpr int kMaxSteps = 64;     // conv MMA K-steps (32 B) per channel group
constexpr int kTileH = 16;        // conv: output rows per tile (one 8-row core group each)
constexpr int kTileW = 8;         // conv: output columns per tile
// Fused max pool: a 16x8 conv tile at origin (14*th - 1, 6*tw - 1) holds
// every 3x3/s2 window of a 7x3 block of pooled outputs.
constexpr int kPoolRows = 7, kPoolCols = 3;  // pooled outputs per 16 x 8 conv tile (3x3/s2 windows)
constexpr int kPoolPix = kPoolRows * kPoolCols;
// Per epilogue set: the pooled int32 accumulators of one tile pair
// ([tile][pooled pixel][64 channels]), staged for the vectorised epilogue.
// The second tile starts 16 words further on, so the two half-warps that
// write one pixel row of each tile hit different banks.
constexpr int kPoolTileWords = kPoolPix * 64 + 16;
constexpr uint32_t kPoolStageBytes = ((2 * kPoolTileWords * 4) + 1023u) & ~1023u;

struct EpiParams {
  void* out;
  int out_kind;  // 0 s32, 1 f32, 2 f16, 3 s8
  int relu;
  const float* alpha;
  float alpha_scalar;
  const float* beta;
  const float* residual;
  long long res_ld;
  float out_scale;
  int qn, qp;
  float* aux;
  long long aux_ld;
  long long s_img, s_pix, s_ch;  // output element strides
  int n_total;                   // valid columns
  int acc_fits_22;               // host-proven |acc| < 2^22: no per-value range check
  int vec16;                     // host-proven: every 16-column chunk below n_total is full and
                                 // 16-byte aligned in out, alpha, beta, residual and aux
  int v8;                        // host-proven (with vec16): the float32 residual, aux and float32
                                 // out chunks are 32-byte aligned (256-bit accesses)
};

// 32-byte global accesses (four float pairs).
__device__ __forceinline__ void ldg256(const float* p, uint64_t& a, uint64_t& b, uint64_t& c, uint64_t& d) {
  asm volatile("ld.global.v4.u64 {%0, %1, %2, %3}, [%4];" : "=l"(a), "=l"(b), "=l"(c), "=l"(d) : "l"(p));
}
__device__ __forceinline__ void stg256(float* p, uint64_t a, uint64_t b, uint64_t c, uint64_t d) {
  asm volatile("st.global.v4.u64 [%0], {%1, %2, %3, %4};" ::"l"(p), "l"(a), "l"(b), "l"(c), "l"(d) : "memory");
}

struct ConvParams {
  int ho, wo;              // output size
  int tiles_h, tiles_w;    // tiles per image
  int n_slots;             // halo sub-tiles (stride phases) in use
  int cg;                  // channel-group width in bytes (16, 32, 64 or 128) = halo pixel pitch
  uint32_t a_layout;       // operand layout of the halo: swizzle matching cg (none for 16)
  int halo_w, halo_h;      // sub-halo size in pixels
  uint32_t slot_bytes;     // bytes per sub-halo (1024-aligned)
  uint32_t halo_bytes;     // 1024-aligned bytes per halo stage (pooled conv: a tile pair)
  uint32_t tile_halo_bytes;  // pooled conv: offset of the pair's second tile in a halo stage
  uint32_t halo_tx_bytes;  // bytes the TMA loads of one stage deliver
  int slot_qh[4], slot_qw[4];  // per slot: TMA start offset in phase-view units
  int wc_bytes;            // > 0: the halo map merges W and C (16-byte pixels, stride 1, one
                           //    channel group) into one dimension, so one box row is a whole
                           //    halo row; the TMA x coordinate is then pixel * wc_bytes
  int kb_per_group;
  uint32_t ab_off;         // smem offset of the epilogue's alpha / beta copies (0: read from global)
  int ab_pitch;            // floats from the alpha copy to the beta copy
  int tail_steps;          // real 32-byte K-steps in a group's last k-block (1..4)
  int pool;                // 1: fused 3x3/s2/p1 max pool (tiles overlap by one row/column)
  int pack2;               // 1: a tile holds two images' 8x8 outputs (stride 1, outputs <= 8x8):
                           //    the halo interleaves the images row by row, MMA row group g is
                           //    output row g / 2 of image 2 * tile + g % 2
  int n;                   // images
  int pho, pwo;            // pooled output size
  uint32_t pool_off;       // pooled conv: smem offset of the per-set output staging (kPoolStageBytes each)
  int extra_set;           // 64-channel conv, resident weights: the unpack warps drain a fifth buffer
  uint32_t dtab_off;       // resident weights: smem offset of the MMA descriptor table
                           // ((A, B) pairs per halo stage, channel group and issued K-step)
  // A-operand descriptor of each 32-byte K-step relative to the halo stage
  // base (start address = offset inside the stage; add stage_addr >> 4).
  uint64_t step_desc[kMaxSteps];
};

struct KParams {
  int M, N;
  int num_kb;        // k-blocks per tile
  int tiles_m, tiles_n;
  int stages;        // operand pipeline depth
  int halo_stages;   // conv halo pipeline depth
  uint32_t a_off, b_off, bp_off, h_off;  // smem region offsets (from 1024-aligned base)
  uint32_t a_stage_bytes, b_stage_bytes, bp_stage_bytes;
  uint32_t tx_bytes;  // TMA bytes per operand stage
  int pk_stages, b8_stages;  // W4 GEMM: packed-weight and int8-weight ring depths
  int k_splits, kb_per_split;  // W4 GEMM split-K: units are (tile, k-range)
  int* ws;                     // split-K: int32 partial sums, [M, ws_ld], zeroed before the launch
  long long ws_ld;
  int b_resident;     // conv, one n-tile: all weight k-blocks stay in smem
  uint32_t bres_tx_bytes;
  uint32_t tmem_cols;
  unsigned* err;
  EpiParams epi;
  ConvParams conv;
};

// ----------------------------- epilogue ------------------------------------
// Exact int32 -> float32 (round to nearest even) without the conversion
// unit for |a| < 2^22: 1.5*2^23 + a is exact in float32, then subtract.
__device__ __forceinline__ float i2f_exact(int a) {
  if (__builtin_expect(static_cast<unsigned>(a + 0x400000) < 0x800000u, 1))
    return __fsub_rn(__int_as_float(a + 0x4B400000), 12582912.0f);
  return __int2float_rn(a);
}

// LSQ code clamp(rint(y / s), qn, qp) with IEEE division semantics.
// t = fl(y * fl(1/s)) differs from fl(y/s) by at most |y/s| * 3.1 * 2^-24
// (< 6.1e-5 for |t| < 256), so rint(t) == rint(fl(y/s)) unless t lies
// within that distance of a half-integer; inside a 2^-12 guard band the
// exact quotient is computed. |t| >= 256 always clamps. The final float ->
// int uses 1.5*2^23 (round to nearest even, exact after the clamp).
__device__ __forceinline__ int lsq_code(float y, float s, float rs, float qnf, float qpf) {
  float t = __fmul_rn(y, rs);
  if (fabsf(t) < 256.0f) {
    const float rt = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);
    if (fabsf(fabsf(__fsub_rn(t, rt)) - 0.5f) < 2.44140625e-4f) t = __fdiv_rn(y, s);
  }
  t = fminf(fmaxf(t, qnf), qpf);
  return __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
}

// Guard-band fix-up of one fast quotient t = fl(y * fl(1/s)): returns the
// exact fl(y / s) when t is within 2^-12 of a half-integer, else t.
__device__ __forceinline__ float lsq_guard(float y, float t, float s) {
  if (fabsf(t) < 256.0f) {
    const float rt = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);
    if (fabsf(fabsf(__fsub_rn(t, rt)) - 0.5f) < 2.44140625e-4f) return __fdiv_rn(y, s);
  }
  return t;
}

struct EpiConsts {
  float rs, qnf, qpf;
  bool relu_in_clamp;  // s8 output, qn >= 0, no float32 side output: the clamp is the ReLU
};

// Packed float32 pairs (add/mul.rn.f32x2: two independent IEEE round-to-
// nearest operations, bit-identical to the scalar forms).
__device__ __forceinline__ uint64_t fpair(float lo, float hi) {
  return uint64_t(__float_as_uint(lo)) | (uint64_t(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float flo(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float fhi(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Common-case epilogue for 16 contiguous columns (aligned vectors, NHWC /
// row-major output): the same arithmetic as epilogue16, on float pairs.
// 16 bytes from shared memory.
__device__ __forceinline__ ulonglong2 lds128(const float* p) {
  ulonglong2 v;
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "r"(smem_u32(p)));
  return v;
}

// kSmemAB: sa / sb, when non-null, are shared-memory copies of alpha / beta
// read in place of e.alpha / e.beta (same values, indexed alike).
template <bool kSmemAB>
__device__ __forceinline__ void epilogue16_fast(const EpiParams& e, const EpiConsts& k, const uint32_t* acc, int n,
                                                long long out_off, long long prow, const float* sa,
                                                const float* sb) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t magic2 = fpair(kMagic, kMagic), neg_magic2 = fpair(-kMagic, -kMagic);
  uint64_t y[8];
  bool small = e.acc_fits_22 != 0;
  if (!small) {
    uint32_t oor = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) oor |= (acc[i] + 0x400000u) & 0xFF800000u;
    small = oor == 0;
  }
  if (small) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      y[j] = add2(uint64_t(acc[2 * j] + 0x4B400000u) | (uint64_t(acc[2 * j + 1] + 0x4B400000u) << 32), neg_magic2);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = fpair(__int2float_rn(int(acc[2 * j])), __int2float_rn(int(acc[2 * j + 1])));
  }
  if (e.alpha) {
    const ulonglong2* a2 = reinterpret_cast<const ulonglong2*>(e.alpha + n);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const ulonglong2 v = (kSmemAB && sa) ? lds128(sa + n + 4 * g) : __ldg(a2 + g);
      y[2 * g] = mul2(y[2 * g], v.x);
      y[2 * g + 1] = mul2(y[2 * g + 1], v.y);
    }
  } else {
    const uint64_t a = fpair(e.alpha_scalar, e.alpha_scalar);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = mul2(y[j], a);
  }
  if (e.beta) {
    const ulonglong2* b2 = reinterpret_cast<const ulonglong2*>(e.beta + n);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const ulonglong2 v = (kSmemAB && sb) ? lds128(sb + n + 4 * g) : __ldg(b2 + g);
      y[2 * g] = add2(y[2 * g], v.x);
      y[2 * g + 1] = add2(y[2 * g + 1], v.y);
    }
  }
  if (e.residual) {
    const float* rp = e.residual + prow * e.res_ld + n;
    if (e.v8) {
      uint64_t r[8];
      ldg256(rp, r[0], r[1], r[2], r[3]);
      ldg256(rp + 8, r[4], r[5], r[6], r[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = add2(y[j], r[j]);
    } else {
      const ulonglong2* r2 = reinterpret_cast<const ulonglong2*>(rp);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const ulonglong2 v = r2[g];
        y[2 * g] = add2(y[2 * g], v.x);
        y[2 * g + 1] = add2(y[2 * g + 1], v.y);
      }
    }
  }
  if (e.relu && !k.relu_in_clamp) {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = fpair(fmaxf(flo(y[j]), 0.0f), fmaxf(fhi(y[j]), 0.0f));
  }
  if (e.aux) {
    float* ap = e.aux + prow * e.aux_ld + n;
    if (e.v8) {
      stg256(ap, y[0], y[1], y[2], y[3]);
      stg256(ap + 8, y[4], y[5], y[6], y[7]);
    } else {
      ulonglong2* d2 = reinterpret_cast<ulonglong2*>(ap);
#pragma unroll
      for (int g = 0; g < 4; ++g) d2[g] = make_ulonglong2(y[2 * g], y[2 * g + 1]);
    }
  }
  if (e.out_kind == 1) {
    float* op = static_cast<float*>(e.out) + out_off;
    if (e.v8) {
      stg256(op, y[0], y[1], y[2], y[3]);
      stg256(op + 8, y[4], y[5], y[6], y[7]);
    } else {
      ulonglong2* d2 = reinterpret_cast<ulonglong2*>(op);
#pragma unroll
      for (int g = 0; g < 4; ++g) d2[g] = make_ulonglong2(y[2 * g], y[2 * g + 1]);
    }
    return;
  }
  if (e.out_kind == 2) {
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      w[j] = uint32_t(__half_as_ushort(__float2half_rn(flo(y[j])))) |
             (uint32_t(__half_as_ushort(__float2half_rn(fhi(y[j])))) << 16);
    uint4* d4 = reinterpret_cast<uint4*>(static_cast<__half*>(e.out) + out_off);
    d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
    return;
  }
  // LSQ codes: t = y * fl(1/s); guard band -> exact quotient (see lsq_code);
  // clamp; the low byte of the 1.5*2^23-biased float is the int8 code.
  const uint64_t rs2 = fpair(k.rs, k.rs);
  uint64_t t[8];
  bool slow = false;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    t[j] = mul2(y[j], rs2);
    const uint64_t rt = add2(add2(t[j], magic2), neg_magic2);
    const uint64_t d = add2(t[j], rt ^ 0x8000000080000000ull);  // t - rint(t)
    // Near-ties only; lsq_guard itself skips |t| >= 256, whose codes saturate.
    slow |= fabsf(flo(d)) > 0.49975586f;
    slow |= fabsf(fhi(d)) > 0.49975586f;
  }
  if (slow) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      t[j] = fpair(lsq_guard(flo(y[j]), flo(t[j]), e.out_scale), lsq_guard(fhi(y[j]), fhi(t[j]), e.out_scale));
  }
  uint32_t b[16];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint64_t c = add2(fpair(fminf(fmaxf(flo(t[j]), k.qnf), k.qpf), fminf(fmaxf(fhi(t[j]), k.qnf), k.qpf)),
                            magic2);
    b[2 * j] = uint32_t(c);
    b[2 * j + 1] = uint32_t(c >> 32);
  }
  uint4 w;
  w.x = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
  w.y = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
  w.z = __byte_perm(__byte_perm(b[8], b[9], 0x0040), __byte_perm(b[10], b[11], 0x0040), 0x5410);
  w.w = __byte_perm(__byte_perm(b[12], b[13], 0x0040), __byte_perm(b[14], b[15], 0x0040), 0x5410);
  *reinterpret_cast<uint4*>(static_cast<int8_t*>(e.out) + out_off) = w;
}

// Applies the fused epilogue to 16 accumulators (columns n .. n+15) of one
// output row; all indexing is static so nothing spills to local memory.
// kSmemAB: sa / sb (optional) are shared-memory copies of alpha / beta for
// the vector path (16-byte aligned at every multiple of 16 columns).
template <bool kSmemAB = false>
__device__ __forceinline__ void epilogue16(const EpiParams& e, const EpiConsts& k, const uint32_t* acc, int n,
                                           long long out_off, long long prow, const float* sa = nullptr,
                                           const float* sb = nullptr) {
  if (e.vec16) {
    if (n < e.n_total) epilogue16_fast<kSmemAB>(e, k, acc, n, out_off, prow, sa, sb);
    return;
  }
  const int ncols = min(16, e.n_total - n);
  if (ncols <= 0) return;
  const bool vec = (ncols == 16) && (e.s_ch == 1);
  if (vec && e.out_kind != 0) {
    const size_t esz = e.out_kind == 1 ? 4 : (e.out_kind == 2 ? 2 : 1);
    const uintptr_t mis =
        (reinterpret_cast<uintptr_t>(static_cast<const char*>(e.out) + out_off * esz)) |
        (e.alpha ? reinterpret_cast<uintptr_t>(e.alpha + n) : 0) | (e.beta ? reinterpret_cast<uintptr_t>(e.beta + n) : 0) |
        (e.residual ? reinterpret_cast<uintptr_t>(e.residual + prow * e.res_ld + n) : 0) |
        (e.aux ? reinterpret_cast<uintptr_t>(e.aux + prow * e.aux_ld + n) : 0);
    if ((mis & 15) == 0) {
      epilogue16_fast<kSmemAB>(e, k, acc, n, out_off, prow, sa, sb);
      return;
    }
  }
  if (e.out_kind == 0) {
    int32_t* dst = static_cast<int32_t*>(e.out) + out_off;
    if (vec && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<int4*>(dst)[i] =
            make_int4(int(acc[4 * i]), int(acc[4 * i + 1]), int(acc[4 * i + 2]), int(acc[4 * i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < ncols) dst[i * e.s_ch] = int(acc[i]);
    }
    return;
  }
  float y[16];
  // int32 -> float32: exact add-and-subtract of 1.5*2^23 unless a value
  // needs more than 22 bits (checked once for all 16).
  uint32_t oor = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) oor |= (acc[i] + 0x400000u) & 0xFF800000u;
  if (oor == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) y[i] = __fsub_rn(__int_as_float(int(acc[i]) + 0x4B400000), 12582912.0f);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) y[i] = __int2float_rn(int(acc[i]));
  }
  // y = y * alpha (+ beta), four columns at a time.
  const bool vec_ab = ncols == 16 && (!e.alpha || (reinterpret_cast<uintptr_t>(e.alpha + n) & 15) == 0) &&
                      (!e.beta || (reinterpret_cast<uintptr_t>(e.beta + n) & 15) == 0);
  if (vec_ab) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float4 av = make_float4(e.alpha_scalar, e.alpha_scalar, e.alpha_scalar, e.alpha_scalar);
      if (e.alpha) av = __ldg(reinterpret_cast<const float4*>(e.alpha + n) + g);
      y[4 * g] = __fmul_rn(y[4 * g], av.x);
      y[4 * g + 1] = __fmul_rn(y[4 * g + 1], av.y);
      y[4 * g + 2] = __fmul_rn(y[4 * g + 2], av.z);
      y[4 * g + 3] = __fmul_rn(y[4 * g + 3], av.w);
      if (e.beta) {
        const float4 bv = __ldg(reinterpret_cast<const float4*>(e.beta + n) + g);
        y[4 * g] = __fadd_rn(y[4 * g], bv.x);
        y[4 * g + 1] = __fadd_rn(y[4 * g + 1], bv.y);
        y[4 * g + 2] = __fadd_rn(y[4 * g + 2], bv.z);
        y[4 * g + 3] = __fadd_rn(y[4 * g + 3], bv.w);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float av = (e.alpha && i < ncols) ? __ldg(e.alpha + n + i) : e.alpha_scalar;
      y[i] = __fmul_rn(y[i], av);
      if (e.beta) y[i] = __fadd_rn(y[i], i < ncols ? __ldg(e.beta + n + i) : 0.0f);
    }
  }
  if (e.residual) {
    const float* res = e.residual + prow * e.res_ld + n;
    if (ncols == 16 && (reinterpret_cast<uintptr_t>(res) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(res + 4 * i);
        y[4 * i] = __fadd_rn(y[4 * i], v.x);
        y[4 * i + 1] = __fadd_rn(y[4 * i + 1], v.y);
        y[4 * i + 2] = __fadd_rn(y[4 * i + 2], v.z);
        y[4 * i + 3] = __fadd_rn(y[4 * i + 3], v.w);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < ncols) y[i] = __fadd_rn(y[i], res[i]);
    }
  }
  if (e.relu) {
#pragma unroll
    for (int i = 0; i < 16; ++i) y[i] = fmaxf(y[i], 0.0f);
  }
  if (e.aux) {
    float* dst = e.aux + prow * e.aux_ld + n;
    if (ncols == 16 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4*>(dst)[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < ncols) dst[i] = y[i];
    }
  }
  if (e.out_kind == 1) {
    float* dst = static_cast<float*>(e.out) + out_off;
    if (vec && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4*>(dst)[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < ncols) dst[i * e.s_ch] = y[i];
    }
  } else if (e.out_kind == 2) {
    __half* dst = static_cast<__half*>(e.out) + out_off;
    if (vec && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = uint32_t(__half_as_ushort(__float2half_rn(y[2 * i]))) |
               (uint32_t(__half_as_ushort(__float2half_rn(y[2 * i + 1]))) << 16);
      reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
      reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < ncols) dst[i * e.s_ch] = __float2half_rn(y[i]);
    }
  } else {
    int8_t* dst = static_cast<int8_t*>(e.out) + out_off;
    // Codes clamp(rint(y / s)): multiply by fl(1/s); the exact quotient is
    // taken only for values inside the rounding guard band (see lsq_code),
    // decided for all 16 at once so the common path has no branches.
    float t[16];
    bool slow = false;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      t[i] = __fmul_rn(y[i], k.rs);
      const float rt = __fsub_rn(__fadd_rn(t[i], 12582912.0f), 12582912.0f);
      slow |= (fabsf(t[i]) < 256.0f) & (fabsf(fabsf(__fsub_rn(t[i], rt)) - 0.5f) < 2.44140625e-4f);
    }
    if (slow) {
#pragma unroll
      for (int i = 0; i < 16; ++i) t[i] = lsq_guard(y[i], t[i], e.out_scale);
    }
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float c = fminf(fmaxf(t[i], k.qnf), k.qpf);
      w[i >> 2] |= (uint32_t(__float_as_int(__fadd_rn(c, 12582912.0f)) - 0x4B400000) & 0xFFu) << (8 * (i & 3));
    }
    if (vec && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < ncols) dst[i * e.s_ch] = int8_t((w[i >> 2] >> (8 * (i & 3))) & 0xFFu);
    }
  }
}

// Conv tiles are split into contiguous per-CTA ranges [conv_tile_begin(b),
// conv_tile_begin(b + 1)): a CTA's consecutive tiles are spatial neighbours,
// and every role steps its tile coordinates with ConvTile::next instead of
// dividing (a single-thread control loop pays for each instruction).
__device__ __forceinline__ int conv_tile_begin(int total, int b, int nb) {
  return int((long long)total * b / nb);
}

struct ConvTile {
  int nt, tw, th, img;  // n-tile, tile column, tile row, image (image pair for two-image tiles)
  __device__ __forceinline__ void init(const KParams& p, int t) {
    const int mt = t / p.tiles_n;
    nt = t - mt * p.tiles_n;
    const int per_img = p.conv.tiles_h * p.conv.tiles_w;
    img = mt / per_img;
    const int rem = mt - img * per_img;
    th = rem / p.conv.tiles_w;
    tw = rem - th * p.conv.tiles_w;
  }
  __device__ __forceinline__ void next(const KParams& p) {
    if (++nt == p.tiles_n) {
      nt = 0;
      if (++tw == p.conv.tiles_w) {
        tw = 0;
        if (++th == p.conv.tiles_h) {
          th = 0;
          ++img;
        }
      }
    }
  }
  // Moves to tile t, `step` tiles on from the current one (next() for a step of one).
  __device__ __forceinline__ void advance(const KParams& p, int t, int step) {
    if (step == 1)
      next(p);
    else
      init(p, t);
  }
  // Output addressing of row m (0..127) of this tile; false outside the output.
  __device__ __forceinline__ bool row(const KParams& p, int m, long long& out_off, long long& prow) const {
    const ConvParams& c = p.conv;
    int im, oh, ow;
    if (c.pack2) {
      im = 2 * img + ((m >> 3) & 1);
      oh = m >> 4;
      ow = m & 7;
    } else {
      im = img;
      oh = th * kTileH + (m >> 3);
      ow = tw * kTileW + (m & 7);
    }
    const long long pix = (long long)oh * c.wo + ow;
    out_off = (long long)im * p.epi.s_img + pix * p.epi.s_pix;
    prow = (long long)im * c.ho * c.wo + pix;
    return im < c.n && oh < c.ho && ow < c.wo;
  }
};

// Bounded wait of a whole warp: lane 0 polls, the warp gets the result.
template <bool kIdle>
__device__ __forceinline__ bool warp_wait(int lane, uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait_t<kIdle>(bar, parity, abort_flag) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Maps (tile m index, row within tile) to output addressing.
template <bool kConv>
__device__ __forceinline__ bool row_coords(const KParams& p, int mt, int m, long long& out_off,
                                           long long& prow) {
  if constexpr (!kConv) {
    const int row = mt * kBM + m;
    out_off = (long long)row * p.epi.s_pix;
    prow = row;
    return row < p.M;
  } else {
    const ConvParams& c = p.conv;
    if (c.pack2) {
      const int img = 2 * mt + ((m >> 3) & 1), oh = m >> 4, ow = m & 7;
      const long long pix = (long long)oh * c.wo + ow;
      out_off = (long long)img * p.epi.s_img + pix * p.epi.s_pix;
      prow = (long long)img * c.ho * c.wo + pix;
      return img < c.n && oh < c.ho && ow < c.wo;
    }
    const int per_img = c.tiles_h * c.tiles_w;
    const int img = mt / per_img;
    const int rem = mt - img * per_img;
    const int th = rem / c.tiles_w;
    const int tw = rem - th * c.tiles_w;
    const int oh = th * kTileH + (m >> 3);
    const int ow = tw * kTileW + (m & 7);
    const long long pix = (long long)oh * c.wo + ow;
    out_off = (long long)img * p.epi.s_img + pix * p.epi.s_pix;
    prow = (long long)img * c.ho * c.wo + pix;
    return oh < c.ho && ow < c.wo;
  }
}

// Fused 3x3/s2/p1 max pool, channel-major accumulators. In the pooled
// stem's M = 64 MMA the accumulator rows are output channels and the columns
// the 128 conv pixels of a 16 x 8 tile (column = row * 8 + col), and each
// TMEM buffer holds two tiles: tile 0 of the pair in lanes 0-15 of every
// 32-lane quadrant, tile 1 in lanes 16-31. The thread of lane l in quadrant q
// therefore owns channel 16 q + (l & 15) of tile (l >> 4) and pools it in
// registers: per conv row, the max (or min) of the three columns of each
// pooled column, then of the three rows of each pooled row. The epilogue is
// increasing in acc where alpha >= 0 and decreasing where alpha < 0, so the
// channel's alpha picks max or min (`use_max`) and the pooled accumulator is
// the one the epilogue then maps. Conv pixels outside the image take the
// value of their nearest in-image neighbour of the same window (the window
// centre is always inside), which leaves max and min unchanged. The pooled
// accumulators go to the set's staging area (sacc: [pooled pixel][64
// channels] of this lane's tile). `valid` is false for the lanes of a missing
// second tile; every lane still takes part in the warp-wide TMEM loads.
__device__ __forceinline__ void pool_channel_tile(const KParams& p, uint32_t t_addr, const ConvTile& ct, bool valid,
                                                  int ch, bool use_max, int* sacc) {
  const ConvParams& c = p.conv;
  const int oh0 = ct.th * (2 * kPoolRows) - 1, ow0 = ct.tw * (2 * kPoolCols) - 1;
  const int right_from = c.wo - ow0;   // first tile column outside the image
  const int bottom_from = c.ho - oh0;  // first tile row outside the image
  // Max pooling of the negated accumulators gives the min: one code path.
  const int sgn = use_max ? 0 : -1;
  int ev[kPoolCols], od[kPoolCols];  // pooled-column values of the last even / odd row
#pragma unroll
  for (int j = 0; j < kPoolCols; ++j) ev[j] = od[j] = 0;
#pragma unroll
  for (int i2 = 0; i2 < kTileH / 4; ++i2) {  // four conv rows (two 16-column loads) per TMEM wait
    uint32_t va[16], vb[16];
    tmem_ld16(t_addr + 32 * i2, va);
    tmem_ld16(t_addr + 32 * i2 + 16, vb);
    tmem_ld_wait();
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const uint32_t* v = s4 < 2 ? va : vb;
      const int s2 = s4 & 1;
      const int r = 4 * i2 + s4;
      if (r > 2 * kPoolRows) break;  // rows 0 .. 14 feed the 7 pooled rows
      int x[kTileW];
#pragma unroll
      for (int cc = 0; cc < kTileW; ++cc) x[cc] = (int(v[kTileW * s2 + cc]) ^ sgn) - sgn;
      if (ow0 < 0) x[0] = x[1];
      if (right_from < kTileW) {
#pragma unroll
        for (int cc = 1; cc < kTileW; ++cc)
          if (cc >= right_from) x[cc] = x[cc - 1];
      }
      int hx[kPoolCols];
#pragma unroll
      for (int j = 0; j < kPoolCols; ++j) hx[j] = __vimax3_s32(x[2 * j], x[2 * j + 1], x[2 * j + 2]);
      if (r >= bottom_from) {  // below the image: repeat the row above
#pragma unroll
        for (int j = 0; j < kPoolCols; ++j) hx[j] = (r & 1) ? ev[j] : od[j];
      }
      if (r & 1) {
#pragma unroll
        for (int j = 0; j < kPoolCols; ++j) {
          if (r == 1 && oh0 < 0) ev[j] = hx[j];  // row 0 lies above the image: row 1 stands in for it
          od[j] = hx[j];
        }
        continue;
      }
      if (r >= 2 && valid) {
#pragma unroll
        for (int j = 0; j < kPoolCols; ++j)
          sacc[((r / 2 - 1) * kPoolCols + j) * 64 + ch] = (__vimax3_s32(ev[j], od[j], hx[j]) ^ sgn) - sgn;
      }
#pragma unroll
      for (int j = 0; j < kPoolCols; ++j) ev[j] = hx[j];
    }
  }
}

// Epilogue and stores of a staged tile pair. Thread tid takes channel quad
// tid & 15 (alpha a4 / beta b4 are that quad's) of pooled pixels
// (tid >> 4) + 8 i of both tiles: float32 values (aux, or out for float32
// output) and int8 codes stored as one vector each. The arithmetic is
// epilogue16_fast's on float pairs (bit-identical to the scalar forms).
__device__ __forceinline__ void pool_store_pair(const KParams& p, const EpiConsts& k, const int* sacc,
                                                const ConvTile& ct0, const ConvTile& ct1, bool has1, int tid,
                                                ulonglong2 a2, ulonglong2 b2) {
  const ConvParams& c = p.conv;
  const EpiParams& e = p.epi;
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t magic2 = fpair(kMagic, kMagic), neg_magic2 = fpair(-kMagic, -kMagic);
  const uint64_t rs2 = fpair(k.rs, k.rs);
  const int quad = tid & 15;
  if (4 * quad >= e.n_total) return;
  const int ch = 4 * quad;
#pragma unroll 1
  for (int it = tid >> 4; it < (has1 ? 2 : 1) * kPoolPix; it += 8) {
    const int h = it >= kPoolPix ? 1 : 0, px = it - h * kPoolPix;
    const ConvTile& ct = h ? ct1 : ct0;
    const int pr_l = px / kPoolCols, pc_l = px - pr_l * kPoolCols;
    const int pr = ct.th * kPoolRows + pr_l, pc = ct.tw * kPoolCols + pc_l;
    if (pr >= c.pho || pc >= c.pwo) continue;
    const int4 acc = *reinterpret_cast<const int4*>(sacc + h * kPoolTileWords + px * 64 + ch);
    // Float pairs, as in epilogue16_fast: exact int32 -> float32 for |acc| < 2^22.
    uint64_t y[2];
    if (e.acc_fits_22) {
      y[0] = add2(uint64_t(uint32_t(acc.x) + 0x4B400000u) | (uint64_t(uint32_t(acc.y) + 0x4B400000u) << 32), neg_magic2);
      y[1] = add2(uint64_t(uint32_t(acc.z) + 0x4B400000u) | (uint64_t(uint32_t(acc.w) + 0x4B400000u) << 32), neg_magic2);
    } else {
      y[0] = fpair(i2f_exact(acc.x), i2f_exact(acc.y));
      y[1] = fpair(i2f_exact(acc.z), i2f_exact(acc.w));
    }
    y[0] = mul2(y[0], a2.x);
    y[1] = mul2(y[1], a2.y);
    if (e.beta) {
      y[0] = add2(y[0], b2.x);
      y[1] = add2(y[1], b2.y);
    }
    if (e.relu) {
      y[0] = fpair(fmaxf(flo(y[0]), 0.0f), fmaxf(fhi(y[0]), 0.0f));
      y[1] = fpair(fmaxf(flo(y[1]), 0.0f), fmaxf(fhi(y[1]), 0.0f));
    }
    const long long prow = ((long long)ct.img * c.pho + pr) * c.pwo + pc;
    if (e.aux) *reinterpret_cast<ulonglong2*>(e.aux + prow * e.aux_ld + ch) = make_ulonglong2(y[0], y[1]);
    if (e.out_kind == 3) {
      // LSQ codes as in epilogue16_fast: t = y * fl(1/s), exact quotient near ties.
      uint64_t t[2];
      bool slow = false;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        t[j] = mul2(y[j], rs2);
        const uint64_t rt = add2(add2(t[j], magic2), neg_magic2);
        const uint64_t d = add2(t[j], rt ^ 0x8000000080000000ull);
        slow |= fabsf(flo(d)) > 0.49975586f;
        slow |= fabsf(fhi(d)) > 0.49975586f;
      }
      if (slow) {
#pragma unroll
        for (int j = 0; j < 2; ++j)
          t[j] = fpair(lsq_guard(flo(y[j]), flo(t[j]), e.out_scale), lsq_guard(fhi(y[j]), fhi(t[j]), e.out_scale));
      }
      uint32_t b[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint64_t cq = add2(fpair(fminf(fmaxf(flo(t[j]), k.qnf), k.qpf), fminf(fmaxf(fhi(t[j]), k.qnf), k.qpf)),
                                 magic2);
        b[2 * j] = uint32_t(cq);
        b[2 * j + 1] = uint32_t(cq >> 32);
      }
      *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(e.out) + prow * e.s_pix + ch) =
          __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
    } else if (e.out_kind == 1) {
      *reinterpret_cast<ulonglong2*>(static_cast<float*>(e.out) + prow * e.s_pix + ch) = make_ulonglong2(y[0], y[1]);
    }
  }
}

// ------------------------------ kernel -------------------------------------
// kPool (conv, 8-bit weights, <= 64 channels, resident weights): the fused
// 3x3/s2 max pool, on M = 64 MMAs with the weights as the A operand (rows =
// output channels) and the tile's 128 conv pixels as B; two tiles share each
// 128-column TMEM buffer (lanes 0-15 / 16-31 of every quadrant).
template <int BN, bool kInt4, bool kConv, bool kPool = false>
__global__ void __launch_bounds__(Roles<kConv>::kThreads, 1)
    w4a8_mma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmH0, const __grid_constant__ CUtensorMap tmH1,
                    const __grid_constant__ CUtensorMap tmH2, const __grid_constant__ CUtensorMap tmH3,
                    const __grid_constant__ KParams p) {
  constexpr int kEpiWarps = Roles<kConv>::kEpiWarps;
  constexpr int kUnpackWarp0 = Roles<kConv>::kUnpackWarp0;
  constexpr int kUnpackThreads = Roles<kConv>::kUnpackWarps * 32;
  constexpr int kUnpackGroups = 2;  // unpack warp groups on alternate k-blocks
  static_assert(!kPool || (kConv && BN == 64 && !kInt4), "the pooled conv: 8-bit weights, 64 channels");
  constexpr int kNB = kPool ? 4 : acc_buffers(BN, kConv);  // accumulator buffers = epilogue warp sets
  constexpr int kSetWarps = kEpiWarps / kNB;               // warps per set (a multiple of 4)
  constexpr int kSlices = kSetWarps / 4;                   // column slices per TMEM lane quadrant
  constexpr uint32_t kBufCols = kPool ? kBM : BN;          // TMEM columns per buffer (kPool: 128 pixels)
  // 64-channel convs with resident weights: the four unpack warps (one per
  // TMEM quadrant) are free once the weights are expanded (or from the start
  // with 8-bit weights) and drain a fifth accumulator buffer.
  constexpr bool kExtra = kConv && BN == 64 && !kPool;
  static_assert(!kExtra || (kNB == 4 && Roles<kConv>::kUnpackWarps == 4), "fifth set: four unpack warps");
  constexpr uint32_t kTmemCols = (kPool || kExtra) ? 512u : tmem_columns(BN, kConv);
  const int nb = (kExtra && p.conv.extra_set) ? kNB + 1 : kNB;  // accumulator buffers in use
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[kMaxStages];
  __shared__ __align__(8) uint64_t bar_ready[kMaxStages];
  __shared__ __align__(8) uint64_t bar_empty[kMaxStages];
  __shared__ __align__(8) uint64_t bar_hfull[kMaxHaloStages];
  __shared__ __align__(8) uint64_t bar_hempty[kMaxHaloStages];
  __shared__ __align__(8) uint64_t bar_tfull[5];
  __shared__ __align__(8) uint64_t bar_tempty[5];
  __shared__ __align__(8) uint64_t bar_drain;
  __shared__ __align__(8) uint64_t bar_bres;    // resident weights landed
  __shared__ __align__(8) uint64_t bar_bready;  // resident weights unpacked
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t base_u32 = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - smem_u32(smem_raw));

  pdl_trigger();  // the next kernel of the stream may launch; it waits for this one in its own pdl_wait
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_ready[s], Roles<kConv>::kUnpackWarps / kUnpackGroups);
      mbar_init(&bar_empty[s], 1);
    }
    for (int s = 0; s < p.halo_stages; ++s) {
      mbar_init(&bar_hfull[s], 1);
      mbar_init(&bar_hempty[s], 1);
    }
    for (int b = 0; b < nb; ++b) {
      mbar_init(&bar_tfull[b], 1);
      mbar_init(&bar_tempty[b], kSetWarps * 32);
    }
    mbar_init(&bar_drain, 1);
    mbar_init(&bar_bres, 1);
    mbar_init(&bar_bready, Roles<kConv>::kUnpackWarps);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    if constexpr (!kConv) {
      tma_prefetch_desc(&tmA);
    } else {
      tma_prefetch_desc(&tmH0);
      if (p.conv.n_slots > 1) tma_prefetch_desc(&tmH1);
      if (p.conv.n_slots > 2) tma_prefetch_desc(&tmH2);
      if (p.conv.n_slots > 3) tma_prefetch_desc(&tmH3);
    }
  }
  if (kConv && warp == 2) {
    // Zero the halo buffers once: bytes no box covers stay 0.
    for (uint32_t i = lane * 16; i < p.conv.halo_bytes * p.halo_stages; i += 32 * 16)
      *reinterpret_cast<uint4*>(base + p.h_off + i) = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  // Everything above touched only shared memory, TMEM and the tensor maps;
  // global memory (weights included: a kernel ahead may have written them)
  // is read and written only after the previous kernel has completed.
  pdl_wait();

  const int total_tiles = p.tiles_m * p.tiles_n;
  const int kbpg = kConv ? p.conv.kb_per_group : p.num_kb;

  // Conv with resident weights: this CTA's contiguous tile range. Otherwise
  // tiles blockIdx.x + i * gridDim.x: with streamed weights, every CTA then
  // reads the same weight stages at about the same time, which keeps them in L2.
  const bool contig = kConv && p.b_resident;
  const int t_begin = contig ? conv_tile_begin(total_tiles, blockIdx.x, gridDim.x) : int(blockIdx.x);
  const int t_end = contig ? conv_tile_begin(total_tiles, blockIdx.x + 1, gridDim.x) : total_tiles;
  const int t_step = contig ? 1 : int(gridDim.x);

  if (warp == 0) {
    // ---------------------------- producer ----------------------------------
    if (lane == 0) {
      int s = 0, hs = 0;
      uint32_t ph = 0, hph = 0;
      bool ok = true;
      if (kConv && p.b_resident) {
        mbar_arrive_expect_tx(&bar_bres, p.bres_tx_bytes);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          uint8_t* bdst = base + p.b_off + kb * p.b_stage_bytes;
          if constexpr (kInt4)
            tma_load_2d(bdst + BN * (kBK / 2), &tmW, &bar_bres, kb * (kBK / 2), 0);
          else
            tma_load_2d(bdst, &tmW, &bar_bres, kb * kBK, 0);
        }
      }
      if constexpr (kConv) {
        // Per tile and channel group: one halo window (a 5-D box per stride
        // phase), then, with streamed weights, the group's weight stages.
        const bool resident = p.b_resident != 0, pool = p.conv.pool != 0, pack2 = p.conv.pack2 != 0;
        const int groups = p.num_kb / kbpg, n_slots = p.conv.n_slots;
        const int hstages = p.halo_stages, stages = p.stages;
        const uint32_t htx = p.conv.halo_tx_bytes, hbytes = p.conv.halo_bytes, slot_bytes = p.conv.slot_bytes;
        ConvTile ct;
        ct.init(p, t_begin);
        // One tile's halo window (a 5-D box per stride phase) for channel group g.
        auto issue_halo = [&](uint8_t* hdst, uint64_t* bar, const ConvTile& tc, int g) {
          const int oh0 = pool ? tc.th * (2 * kPoolRows) - 1 : tc.th * kTileH;
          const int ow0 = pool ? tc.tw * (2 * kPoolCols) - 1 : tc.tw * kTileW;
          for (int sl = 0; sl < n_slots; ++sl) {
            const CUtensorMap* m = sl == 0 ? &tmH0 : sl == 1 ? &tmH1 : sl == 2 ? &tmH2 : &tmH3;
            if (pack2)  // map dims (c, group, W, N, H): both images' halo rows, interleaved
              tma_load_5d(hdst + sl * slot_bytes, m, bar, 0, g, ow0 + p.conv.slot_qw[sl], 2 * tc.img,
                          oh0 + p.conv.slot_qh[sl]);
            else if (p.conv.wc_bytes)  // map dims (W * C, 1, 1, H, N)
              tma_load_5d(hdst + sl * slot_bytes, m, bar, (ow0 + p.conv.slot_qw[sl]) * p.conv.wc_bytes, 0, 0,
                          oh0 + p.conv.slot_qh[sl], tc.img);
            else
              tma_load_5d(hdst + sl * slot_bytes, m, bar, 0, g, ow0 + p.conv.slot_qw[sl], oh0 + p.conv.slot_qh[sl],
                          tc.img);
          }
        };
        if (kPool) {
          // Pooled conv (one channel group, resident weights): a halo stage
          // holds a tile pair, one barrier phase for both.
          for (int t = t_begin; ok && t < t_end; t += 2) {
            const int pair = t + 1 < t_end ? 2 : 1;
            if (!mbar_wait_t<true>(&bar_hempty[hs], hph ^ 1, &abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&bar_hfull[hs], htx * uint32_t(pair));
            for (int h = 0; h < pair; ++h) {
              issue_halo(base + p.h_off + hs * hbytes + h * p.conv.tile_halo_bytes, &bar_hfull[hs], ct, 0);
              ct.next(p);
            }
            if (++hs == hstages) { hs = 0; hph ^= 1; }
          }
        }
        for (int t = t_begin; !kPool && ok && t < t_end; t += t_step, ct.advance(p, t, t_step)) {
          int kb = 0;
          for (int g = 0; ok && g < groups; ++g) {
            if (!mbar_wait_t<true>(&bar_hempty[hs], hph ^ 1, &abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&bar_hfull[hs], htx);
            issue_halo(base + p.h_off + hs * hbytes, &bar_hfull[hs], ct, g);
            if (++hs == hstages) { hs = 0; hph ^= 1; }
            if (resident) continue;
            for (int i = 0; i < kbpg; ++i, ++kb) {
              if (!mbar_wait_t<true>(&bar_empty[s], ph ^ 1, &abort_flag)) { ok = false; break; }
              mbar_arrive_expect_tx(&bar_full[s], p.tx_bytes);
              uint8_t* bdst = base + p.b_off + s * p.b_stage_bytes;
              if constexpr (kInt4)
                tma_load_2d(bdst + BN * (kBK / 2), &tmW, &bar_full[s], kb * (kBK / 2), ct.nt * BN);
              else
                tma_load_2d(bdst, &tmW, &bar_full[s], kb * kBK, ct.nt * BN);
              if (++s == stages) { s = 0; ph ^= 1; }
            }
          }
        }
      } else {
        for (int t = t_begin; ok && t < t_end; t += t_step) {
          const int mt = t / p.tiles_n;
          const int nt = t - mt * p.tiles_n;
          for (int kb = 0; ok && kb < p.num_kb; ++kb) {
            if (!mbar_wait(&bar_empty[s], ph ^ 1, &abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&bar_full[s], p.tx_bytes);
            tma_load_2d(base + p.a_off + s * p.a_stage_bytes, &tmA, &bar_full[s], kb * kBK, mt * kBM);
            uint8_t* bdst = base + p.b_off + s * p.b_stage_bytes;
            if constexpr (kInt4)
              tma_load_2d(bdst + BN * (kBK / 2), &tmW, &bar_full[s], kb * (kBK / 2), nt * BN);
            else
              tma_load_2d(bdst, &tmW, &bar_full[s], kb * kBK, nt * BN);
            if (++s == p.stages) { s = 0; ph ^= 1; }
          }
        }
      }
      // Drain: every TMA this thread issued has landed before the CTA exits.
      for (int i = 0; i < p.stages; ++i) {
        const int idx = (s + p.stages - 1 - i) % p.stages;
        const uint32_t par = (idx < s) ? ph : (ph ^ 1);
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(&bar_full[idx], par))
          if (global_timer_ns() - t0 > kWaitLimitNs) { abort_flag = 1; break; }
      }
      if (kConv && p.b_resident) {
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(&bar_bres, 0))
          if (global_timer_ns() - t0 > kWaitLimitNs) { abort_flag = 1; break; }
      }
      for (int i = 0; kConv && i < p.halo_stages; ++i) {
        const int idx = (hs + p.halo_stages - 1 - i) % p.halo_stages;
        const uint32_t par = (idx < hs) ? hph : (hph ^ 1);
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(&bar_hfull[idx], par))
          if (global_timer_ns() - t0 > kWaitLimitNs) { abort_flag = 1; break; }
      }
      if (!ok) atomicOr(p.err, kErrTimeoutProducer);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA ------------------------------------
    constexpr uint32_t idesc = make_idesc_i8(kBM, BN);
    // Descriptor templates (start address 0): the issue loop only adds the
    // stage / halo base.
    const uint64_t sw128_tmpl = make_smem_desc(0, 16, 1024, kLayoutSw128);
    const uint32_t a_stage0 = (base_u32 + p.a_off) >> 4, b_stage0 = (base_u32 + p.b_off) >> 4;
    const uint32_t a_step = p.a_stage_bytes >> 4, b_step = p.b_stage_bytes >> 4;
    if constexpr (kConv) {
      // The whole warp runs the issue loop and one elected lane issues each
      // MMA and commit: a converged warp issues its instructions markedly
      // faster than one lane looping alone while the rest of the warp waits.
      const bool resident = p.b_resident != 0;
      const int groups = p.num_kb / kbpg, hstages = p.halo_stages;
      // Resident weights: the (A, B) descriptor pair of every (halo stage,
      // channel group, K-step) is built once into shared memory, so an MMA
      // costs one 16-byte shared load and its issue. The zero-weight padding
      // steps of a group's last k-block are not issued.
      const int gsteps = (kbpg - 1) * 4 + p.conv.tail_steps;
      ulonglong2* dtab = reinterpret_cast<ulonglong2*>(base + p.conv.dtab_off);
      if (resident) {
        // Pooled conv: "groups" indexes the tile of the pair (one channel group).
        const int per_stage = (kPool ? 2 : groups) * gsteps;
        for (int i = lane; i < hstages * per_stage; i += 32) {
          const int h = i / per_stage, r = i - h * per_stage, g = r / gsteps, j = r - g * gsteps;
          const uint32_t halo_lo =
              (base_u32 + p.h_off + uint32_t(h) * p.conv.halo_bytes + (kPool ? uint32_t(g) * p.conv.tile_halo_bytes : 0u)) >>
              4;
          const uint32_t kb = uint32_t(g * kbpg + (j >> 2));
          dtab[i] = make_ulonglong2(p.conv.step_desc[j] + halo_lo,
                                    sw128_tmpl + (b_stage0 + (kPool ? uint32_t(j >> 2) : kb) * b_step) +
                                        2 * uint32_t(j & 3));
        }
        __syncwarp();
      }
      int hs = 0, buf = 0;
      uint32_t hph = 0, tph = 0;
      bool ok = true;
      if (kPool && resident) {
        // Pooled stem: tiles t, t + 1 of the CTA's range go to one buffer, at
        // TMEM lanes 0 and 16 (M = 64: 16 lanes of each quadrant per tile);
        // operands swapped (A = weights, B = the tile's pixels).
        constexpr uint32_t idesc64 = make_idesc_i8(64, kBM);
        ok = warp_wait<true>(lane, &bar_bres, 0, &abort_flag);
        // Software-pipelined: the next pair's buffer and halo waits run
        // while the tensor core still works through this pair's queued MMAs,
        // and this pair's commits follow them.
        if (ok && t_begin < t_end) {
          ok = warp_wait<true>(lane, &bar_tempty[buf], tph ^ 1, &abort_flag);
          ok = ok && warp_wait<true>(lane, &bar_hfull[hs], hph, &abort_flag);
        }
        for (int t = t_begin; ok && t < t_end; t += 2) {
          tc_fence_after();
          for (int h = 0; h < 2 && t + h < t_end; ++h) {
            const uint32_t d_tmem = tmem_base + buf * kBufCols + (uint32_t(16 * h) << 16);
            const ulonglong2* e = dtab + (hs * 2 + h) * gsteps;
            ulonglong2 d = e[0];
            ulonglong2 dn = e[gsteps > 1 ? 1 : 0];
            mma_i8_ss_elect(d_tmem, d.y, d.x, idesc64, 0u);
            for (int j = 1; j < gsteps; ++j) {
              d = dn;
              dn = e[j + 1 < gsteps ? j + 1 : j];
              mma_i8_ss_elect(d_tmem, d.y, d.x, idesc64, 1u);
            }
          }
          int nbuf = buf + 1, nhs = hs + 1;
          uint32_t ntph = tph, nhph = hph;
          if (nbuf == kNB) { nbuf = 0; ntph ^= 1; }
          if (nhs == hstages) { nhs = 0; nhph ^= 1; }
          if (t + 2 < t_end) {
            ok &= warp_wait<true>(lane, &bar_tempty[nbuf], ntph ^ 1, &abort_flag);
            ok &= warp_wait<true>(lane, &bar_hfull[nhs], nhph, &abort_flag);
          }
          mma_commit_elect(&bar_hempty[hs]);
          mma_commit_elect(&bar_tfull[buf]);
          buf = nbuf;
          tph = ntph;
          hs = nhs;
          hph = nhph;
        }
        mma_commit_elect(&bar_drain);
      } else if (resident) {
        ok = warp_wait<true>(lane, kInt4 ? &bar_bready : &bar_bres, 0, &abort_flag);
        // The inner loops carry no break: a failed wait clears `ok` and sets
        // the CTA's abort flag (so every later wait gives up within a few
        // hundred polls), the tile's remaining MMAs read in-bounds shared
        // memory, and the tile loop stops.
        for (int t = t_begin; ok && t < t_end; t += t_step) {
          if (!warp_wait<true>(lane, &bar_tempty[buf], tph ^ 1, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * BN;
          for (int g = 0; g < groups; ++g) {
            ok &= warp_wait<true>(lane, &bar_hfull[hs], hph, &abort_flag);
            tc_fence_after();
            // The next pair is loaded before the current MMA issues: the MMA
            // asm's memory clobber would otherwise order the load after it
            // and expose its latency once per MMA. (Loading four pairs and
            // then issuing their MMAs back to back measured slower.)
            const ulonglong2* e = dtab + (hs * groups + g) * gsteps;
            ulonglong2 d = e[0];
            ulonglong2 dn = e[gsteps > 1 ? 1 : 0];
            mma_i8_ss_elect(d_tmem, d.x, d.y, idesc, g != 0 ? 1u : 0u);
            for (int j = 1; j < gsteps; ++j) {
              d = dn;
              dn = e[j + 1 < gsteps ? j + 1 : j];
              mma_i8_ss_elect(d_tmem, d.x, d.y, idesc, 1u);
            }
            mma_commit_elect(&bar_hempty[hs]);
            if (++hs == hstages) { hs = 0; hph ^= 1; }
          }
          mma_commit_elect(&bar_tfull[buf]);
          if (++buf == nb) { buf = 0; tph ^= 1; }
        }
        // Drain: all tcgen05 ops of this warp complete before TMEM is freed.
        mma_commit_elect(&bar_drain);
      } else if (lane == 0) {
        // Streamed weights: one lane waits for every weight stage and issues
        // that k-block's four MMAs.
        int s = 0;
        uint32_t ph = 0;
        for (int t = t_begin; ok && t < t_end; t += t_step) {
          if (!mbar_wait_t<true>(&bar_tempty[buf], tph ^ 1, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * BN;
          int kb = 0;
          for (int g = 0; g < groups; ++g) {
            ok &= mbar_wait_t<true>(&bar_hfull[hs], hph, &abort_flag);
            tc_fence_after();
            const uint32_t halo_lo = (base_u32 + p.h_off + hs * p.conv.halo_bytes) >> 4;
            // A k-block's four step descriptors are loaded before its MMAs
            // issue, and the next block's while they issue.
            const uint64_t* sd = p.conv.step_desc;
            uint64_t dn0 = sd[0], dn1 = sd[1], dn2 = sd[2], dn3 = sd[3];
            for (int i = 0; i < kbpg; ++i, ++kb) {
              const uint64_t d0 = dn0 + halo_lo, d1 = dn1 + halo_lo, d2 = dn2 + halo_lo, d3 = dn3 + halo_lo;
              const uint64_t* nx = sd + 4 * min(i + 1, kbpg - 1);
              dn0 = nx[0];
              dn1 = nx[1];
              dn2 = nx[2];
              dn3 = nx[3];
              ok &= mbar_wait_t<true>(kInt4 ? &bar_ready[s] : &bar_full[s], ph, &abort_flag);
              tc_fence_after();
              const uint64_t b_desc0 = sw128_tmpl + (b_stage0 + uint32_t(s) * b_step);
              mma_i8_ss(d_tmem, d0, b_desc0, idesc, kb != 0 ? 1u : 0u);
              mma_i8_ss(d_tmem, d1, b_desc0 + 2, idesc, 1u);
              mma_i8_ss(d_tmem, d2, b_desc0 + 4, idesc, 1u);
              mma_i8_ss(d_tmem, d3, b_desc0 + 6, idesc, 1u);
              mma_commit(&bar_empty[s]);
              if (++s == p.stages) { s = 0; ph ^= 1; }
            }
            mma_commit(&bar_hempty[hs]);
            if (++hs == hstages) { hs = 0; hph ^= 1; }
          }
          mma_commit(&bar_tfull[buf]);
          if (++buf == kNB) { buf = 0; tph ^= 1; }
        }
        mma_commit(&bar_drain);
      }
      if (lane == 0) {
        const unsigned long long w0 = global_timer_ns();
        while (!mbar_try_wait(&bar_drain, 0))
          if (global_timer_ns() - w0 > kWaitLimitNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
        if (!ok) atomicOr(p.err, kErrTimeoutMma);
      }
      __syncwarp();
    } else if (lane == 0) {
      int s = 0, it = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; t += t_step, ++it) {
        const int buf = it % kNB;
        if (!mbar_wait(&bar_tempty[buf], ((it / kNB) & 1) ^ 1, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          ok &= mbar_wait(kInt4 ? &bar_ready[s] : &bar_full[s], ph, &abort_flag);
          tc_fence_after();
          const uint64_t a_desc0 = sw128_tmpl + (a_stage0 + uint32_t(s) * a_step);
          const uint64_t b_desc0 = sw128_tmpl + (b_stage0 + uint32_t(s) * b_step);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_i8_ss(d_tmem, a_desc0 + 2 * j, b_desc0 + 2 * j, idesc, (kb | j) != 0 ? 1u : 0u);
          mma_commit(&bar_empty[s]);
          if (++s == p.stages) { s = 0; ph ^= 1; }
        }
        mma_commit(&bar_tfull[buf]);
      }
      // Drain: all tcgen05 ops of this thread complete before TMEM is freed.
      mma_commit(&bar_drain);
      const unsigned long long w0 = global_timer_ns();
      while (!mbar_try_wait(&bar_drain, 0))
        if (global_timer_ns() - w0 > kWaitLimitNs) { atomicOr(p.err, kErrTimeoutDrain); break; }
      if (!ok) atomicOr(p.err, kErrTimeoutMma);
    }
  } else if (kPool && warp >= 4 && warp < 4 + kEpiWarps) {
    // ------------------------- pooled epilogue -----------------------------
    // Set `set` (one warp per TMEM quadrant) takes the tile pairs of buffer
    // `set`: pairs t_begin + 2 (set + j kNB).
    const int q = warp & 3, set = (warp - 4) / kSetWarps, half = lane >> 4;
    const int ch = 16 * q + (lane & 15);
    const bool ch_ok = ch < p.epi.n_total;
    EpiConsts k;
    k.rs = p.epi.out_kind == 3 ? __frcp_rn(p.epi.out_scale) : 1.0f;
    k.qnf = float(p.epi.qn);
    k.qpf = float(p.epi.qp);
    k.relu_in_clamp = false;
    const float alpha = p.epi.alpha ? (ch_ok ? __ldg(p.epi.alpha + ch) : 0.0f) : p.epi.alpha_scalar;
    const bool use_max = alpha >= 0.0f;
    // This thread's channel quad in the store phase (tid & 15 = lane & 15).
    const int sq4 = 4 * (lane & 15);
    ulonglong2 a2 = make_ulonglong2(fpair(p.epi.alpha_scalar, p.epi.alpha_scalar),
                                    fpair(p.epi.alpha_scalar, p.epi.alpha_scalar));
    ulonglong2 b2 = make_ulonglong2(0ull, 0ull);
    if (sq4 < p.epi.n_total) {
      if (p.epi.alpha) a2 = __ldg(reinterpret_cast<const ulonglong2*>(p.epi.alpha + sq4));
      if (p.epi.beta) b2 = __ldg(reinterpret_cast<const ulonglong2*>(p.epi.beta + sq4));
    }
    const uint32_t t_addr = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(set) * kBufCols;
    uint32_t tph = 0;
    for (int t = t_begin + 2 * set; t < t_end; t += 2 * kNB, tph ^= 1) {
      const int tt = t + half;  // this lane's tile
      const bool has1 = t + 1 < t_end;
      ConvTile ct0, ct1;
      ct0.init(p, t);
      ct1.init(p, has1 ? t + 1 : t);
      const ConvTile& ct = half ? ct1 : ct0;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_idle(&bar_tfull[set], tph, &abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicOr(p.err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      int* stage = reinterpret_cast<int*>(base + p.conv.pool_off + uint32_t(set) * kPoolStageBytes);
      pool_channel_tile(p, t_addr, ct, tt < t_end && ch_ok, ch, use_max, stage + half * kPoolTileWords);
      tc_fence_before();
      mbar_arrive(&bar_tempty[set]);  // the accumulators are in registers / staging now
      bar_sync(2 + set, kSetWarps * 32);
      pool_store_pair(p, k, stage, ct0, ct1, has1, (warp - 4) % kSetWarps * 32 + lane, a2, b2);
      bar_sync(2 + set, kSetWarps * 32);  // the staging area is free for the next pair
    }
  } else if (warp >= 4) {
    if (warp >= kUnpackWarp0) {
      if constexpr (kInt4) {
      // ------------------------------ unpack ---------------------------------
    // ------------------------------ unpack ---------------------------------
    // kUnpackGroups groups of warps take alternate k-blocks, so one group's
    // unpack latency (wait, read, expand, write, proxy fence) overlaps the
    // others'. TMA drops a stage's packed nibbles into the upper half of the
    // int8 rows they expand to. A group first expands rows [0, BN/2), whose
    // targets lie below the packed half, then reads the packed bytes of rows
    // [BN/2, BN), meets at its named barrier (every packed byte of the stage
    // has now been read) and writes those rows over the packed half.
    constexpr int kGT = kUnpackThreads / kUnpackGroups;  // threads per group
    constexpr int kHalf = BN * 4 / kGT;                  // int8 chunks per thread and half
    static_assert(kGT % 64 == 0 && kHalf >= 1, "unpack group shape");
    const int ut = threadIdx.x - kUnpackWarp0 * 32;
    const int ug = ut / kGT, gt = ut % kGT;
    const uint32_t bar_id = 6 + ug;
    // Chunk gt + kGT * j is 16-byte chunk (gt & 7) of int8 row (gt >> 3) + j * kGT / 8;
    // kGT is a multiple of 64, so the swizzle term (row & 7) is the same for all j.
    const uint32_t src0 = BN * (kBK / 2) + gt * 8;
    const uint32_t dst0 = (gt >> 3) * 128 + (((gt & 7) ^ ((gt >> 3) & 7)) << 4);
    bool ok = true;
    const bool resident = kConv && p.b_resident;
    // One lane per warp polls the mbarrier (all 32 polling one word
    // serialises on the shared-memory bank); the shuffle orders the rest of
    // the warp after the observed phase.
    auto wait_warp = [&](uint64_t* bar, uint32_t parity) -> bool {
      int got = 1;
      if (lane == 0) got = mbar_wait_t<kConv>(bar, parity, &abort_flag) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      return got != 0;
    };
    if (resident) ok = bar_and(bar_id, kGT, wait_warp(&bar_bres, 0));
    // Resident weights: one pass over the k-blocks; otherwise one per tile of
    // this CTA's sequence.
    const int t0 = resident ? 0 : t_begin, t1 = resident ? 1 : t_end, ts = resident ? 1 : t_step;
    uint32_t q = 0;  // k-block sequence number of this CTA
    for (int t = t0; ok && t < t1; t += ts) {
      for (int kb = 0; kb < p.num_kb; ++kb, ++q) {
        if (int(q % kUnpackGroups) != ug) continue;
        const uint32_t s = resident ? uint32_t(kb) : q % uint32_t(p.stages);
        if (!resident) {
          if (!bar_and(bar_id, kGT, wait_warp(&bar_full[s], (q / uint32_t(p.stages)) & 1))) { ok = false; break; }
        }
        uint8_t* stage = base + p.b_off + s * p.b_stage_bytes;
        uint2 v[kHalf];
#pragma unroll
        for (int j = 0; j < kHalf; ++j) v[j] = *reinterpret_cast<const uint2*>(stage + src0 + j * kGT * 8);
#pragma unroll
        for (int j = 0; j < kHalf; ++j) {
          uint4 o;
          unpack_nibbles8(v[j].x, o.x, o.y);
          unpack_nibbles8(v[j].y, o.z, o.w);
          *reinterpret_cast<uint4*>(stage + dst0 + j * kGT * 16) = o;
        }
#pragma unroll
        for (int j = 0; j < kHalf; ++j)
          v[j] = *reinterpret_cast<const uint2*>(stage + src0 + (kHalf + j) * kGT * 8);
        bar_sync(bar_id, kGT);
#pragma unroll
        for (int j = 0; j < kHalf; ++j) {
          uint4 o;
          unpack_nibbles8(v[j].x, o.x, o.y);
          unpack_nibbles8(v[j].y, o.z, o.w);
          *reinterpret_cast<uint4*>(stage + dst0 + (kHalf + j) * kGT * 16) = o;
        }
        fence_proxy_async_smem();
        if (resident) continue;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_ready[s]);
      }
    }
    __syncwarp();
    if (resident && ok && lane == 0) mbar_arrive(&bar_bready);
    if (!ok && ut == 0) atomicOr(p.err, kErrTimeoutUnpack);
      }
    }
    if (warp < 4 + kEpiWarps || nb > kNB) {
    // ----------------------------- epilogue --------------------------------
    // Warps 4 + 4 s .. 4 + 4 s + 3 form set s; with a fifth set the unpack
    // warps (after the resident weights are expanded) are set kNB.
    const int q = warp & 3;
    const int set = (warp - 4) / kSetWarps;          // this warp drains buffer `set`
    const int slice = ((warp - 4) % kSetWarps) >> 2;
    const int m = q * 32 + lane;
    EpiConsts k;
    k.rs = p.epi.out_kind == 3 ? __frcp_rn(p.epi.out_scale) : 1.0f;
    k.qnf = float(p.epi.qn);
    k.qpf = float(p.epi.qp);
    k.relu_in_clamp = p.epi.out_kind == 3 && p.epi.qn >= 0 && p.epi.aux == nullptr;
    // Conv: alpha / beta are copied into shared memory once; every 16-column
    // chunk then reads them there instead of making a round trip to L2.
    const float* sa = nullptr;
    const float* sb = nullptr;
    if (kConv && p.conv.ab_off) {
      float* a_s = reinterpret_cast<float*>(base + p.conv.ab_off);
      float* b_s = a_s + p.conv.ab_pitch;
      for (int i = (warp - 4) * 32 + lane; i < p.epi.n_total; i += nb * kSetWarps * 32) {
        if (p.epi.alpha) a_s[i] = p.epi.alpha[i];
        if (p.epi.beta) b_s[i] = p.epi.beta[i];
      }
      bar_sync(8, nb * kSetWarps * 32);
      sa = p.epi.alpha ? a_s : nullptr;
      sb = p.epi.beta ? b_s : nullptr;
    }
    // This warp set takes every nb-th tile of the CTA's sequence (buffer `set`).
    const int buf = set;
    uint32_t tph = 0;
    ConvTile ct;
    if (kConv && t_begin + set * t_step < t_end) ct.init(p, t_begin + set * t_step);
    for (int t = t_begin + set * t_step; t < t_end; t += nb * t_step, tph ^= 1) {
      int mt = 0, nt = 0;
      if constexpr (!kConv) {
        mt = t / p.tiles_n;
        nt = t - mt * p.tiles_n;
      } else {
        nt = ct.nt;
      }
      long long out_off = 0, prow = 0;
      bool valid;
      if constexpr (kConv)
        valid = ct.row(p, m, out_off, prow);
      else
        valid = row_coords<false>(p, mt, m, out_off, prow);
      if (p.epi.residual && valid) {
        // The float32 identity rows of this thread's pixel are pulled into L2
        // while the MMA still works on the tile, so the epilogue's loads hit.
        const char* r = reinterpret_cast<const char*>(p.epi.residual + prow * p.epi.res_ld + nt * BN);
        const int nbytes = 4 * min(BN, p.epi.n_total - nt * BN);
        for (int off = slice * 128; off < nbytes; off += 128 * kSlices)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(r + off));
      }
      int ok = 1;
      if (lane == 0) ok = mbar_wait_idle(&bar_tfull[buf], tph, &abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicOr(p.err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const uint32_t t_addr = tmem_base + (uint32_t(q * 32) << 16) + buf * BN;
      const int c_end = (slice + 1) * (BN / kSlices);
#pragma unroll 1
      for (int c0 = slice * (BN / kSlices); c0 < c_end; c0 += 16) {
        uint32_t acc[16];
        tmem_ld16(t_addr + c0, acc);
        tmem_ld_wait();
        if (c0 + 16 >= c_end) {
          // The last chunk is in registers: the buffer goes back to the MMA
          // before this chunk's epilogue runs.
          tc_fence_before();
          mbar_arrive(&bar_tempty[buf]);
        }
        if (valid) {
          const int n = nt * BN + c0;
          epilogue16<kConv>(p.epi, k, acc, n, out_off + (long long)n * p.epi.s_ch, prow, sa, sb);
        }
      }
      if constexpr (kConv) {
        if (contig) {
          for (int i = 0; i < nb; ++i) ct.next(p);
        } else if (t + nb * t_step < t_end) {
          ct.init(p, t + nb * t_step);
        }
      }
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace w4a8
