// Memory-bound helper kernels around the tensor-core path: LSQ
// quantisation, layout changes, the reference's explicit 3x3 lowering,
// int4 weight reordering and pooling. All quantisation uses IEEE division
// and round-half-to-even: q = clamp(rint(x / s), qn, qp).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "launch.cuh"
#include "w4a8.h"

namespace {

__device__ __forceinline__ int quant1(float x, float scale, int qn, int qp) {
  const int q = __float2int_rn(__fdiv_rn(x, scale));
  return max(qn, min(qp, q));
}

inline int grid_for(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  if (b > (1ll << 20)) b = 1ll << 20;
  return b < 1 ? 1 : int(b);
}

bool q_ok(float scale, int qn, int qp) { return scale > 0.0f && qn >= -128 && qp <= 127 && qn <= qp; }

__global__ void quantize_rows_kernel(const float* __restrict__ x, long long ldx, int8_t* __restrict__ q,
                                     long long ldq, long long rows, int cols, float scale, int qn, int qp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  const long long total = rows * ldq;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / ldq;
    const int k = int(i - r * ldq);
    q[i] = k < cols ? int8_t(quant1(x[r * ldx + k], scale, qn, qp)) : int8_t(0);
  }
}

// x [n, c, h, w] -> y [n, h, w, cp]; one block transposes a 32(c) x 32(hw)
// tile of one image through shared memory.
__global__ void nchw_to_nhwc_q_kernel(const float* __restrict__ x, int8_t* __restrict__ y, int c, int hw,
                                      int cp, float scale, int qn, int qp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  __shared__ int8_t tile[32][33];
  const int img = blockIdx.z;
  const int c0 = blockIdx.y * 32;
  const int p0 = blockIdx.x * 32;
  const float* xi = x + (long long)img * c * hw;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int ch = c0 + i, p = p0 + threadIdx.x;
    int v = 0;
    if (ch < c && p < hw) v = quant1(xi[(long long)ch * hw + p], scale, qn, qp);
    tile[i][threadIdx.x] = int8_t(v);  // channels >= c become the 0 code
  }
  __syncthreads();
  int8_t* yi = y + (long long)img * hw * cp;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int p = p0 + i, ch = c0 + threadIdx.x;
    if (p < hw && ch < cp) yi[(long long)p * cp + ch] = tile[threadIdx.x][i];
  }
}

// Space-to-depth by 2 + quantise: one thread per output pixel.
__global__ void s2d_q_kernel(const float* __restrict__ x, int8_t* __restrict__ y, int n, int c, int h, int w,
                             int cp, float scale, int qn, int qp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  const int ho = h / 2, wo = w / 2;
  const long long total = (long long)n * ho * wo;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int X = int(i % wo);
    const long long t = i / wo;
    const int Y = int(t % ho);
    const int img = int(t / ho);
    int8_t* dst = y + i * cp;
    for (int k = 0; k < cp; k += 16) {
      uint32_t word[4] = {0, 0, 0, 0};
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        const int ch = k + b;  // (dy*2 + dx)*c + cc
        if (ch < 4 * c) {
          const int cc = ch % c, d = ch / c, dy = d >> 1, dx = d & 1;
          const float v = x[(((long long)img * c + cc) * h + 2 * Y + dy) * w + 2 * X + dx];
          word[b >> 2] |= (uint32_t(quant1(v, scale, qn, qp)) & 0xFFu) << (8 * (b & 3));
        }
      }
      *reinterpret_cast<uint4*>(dst + k) = make_uint4(word[0], word[1], word[2], word[3]);
    }
  }
}

// clamp(rint(x / s), qn, qp) without a division per element: t = x * fl(1/s)
// differs from fl(x/s) by at most |x/s| * 3.1 * 2^-24 (< 6.1e-5 for |t| < 256),
// so rint agrees unless t lies within that distance of a half-integer; inside
// a 2^-12 guard band the exact quotient is taken. |t| >= 256 always clamps.
__device__ __forceinline__ int quant_rs(float x, float scale, float rs, float qnf, float qpf) {
  float t = __fmul_rn(x, rs);
  if (fabsf(t) < 256.0f) {
    const float rt = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);
    if (fabsf(fabsf(__fsub_rn(t, rt)) - 0.5f) < 2.44140625e-4f) t = __fdiv_rn(x, scale);
  }
  t = fminf(fmaxf(t, qnf), qpf);
  return __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
}

// Space-to-depth by 2 + quantise, vectorised: a thread makes output pixels
// 2j and 2j + 1 of one row from six coalesced float4 loads (3 channels x 2
// input rows, 4 consecutive columns each). Needs c == 3, cp == 16, w % 4 == 0
// and a 16-byte aligned x. threadIdx.y picks an output row (image * ho + Y)
// of the block and threadIdx.x the column pairs j of that row, so no index
// needs a 64-bit division. The 24 values of a thread are quantised as 12
// float pairs (add/mul.rn.f32x2, bit-identical to the scalar forms) as soon
// as they are loaded; if any t lies within 2^-12 of a half-integer the
// thread reloads its inputs and redoes them through quant_rs's exact path.
// At most 51 registers (5 blocks of 256 per SM): the kernel is bound by the
// loads it keeps in flight.
__device__ __forceinline__ uint64_t s2d_pair(float lo, float hi) {
  return uint64_t(__float_as_uint(lo)) | (uint64_t(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ uint64_t s2d_add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t s2d_mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__global__ void __launch_bounds__(256, 5) s2d_q3_vec_kernel(const float* __restrict__ x, int8_t* __restrict__ y, int n,
                                                         int h, int w, float scale, float rs, int qn, int qp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  const int ho = h / 2, wq = w / 4;  // wq thread columns of two output pixels each
  const int row = int(blockIdx.x * blockDim.y + threadIdx.y);
  if (row >= n * ho) return;
  const int img = row / ho, Y = row - img * ho;
  const float qnf = float(qn), qpf = float(qp);
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t rs2 = s2d_pair(rs, rs), magic2 = s2d_pair(kMagic, kMagic), nmagic2 = s2d_pair(-kMagic, -kMagic);
  const float* xr = x + ((long long)img * 3 * h + 2 * Y) * w;
  int8_t* yr = y + ((long long)row * (w / 2)) * 16;
  for (int j = threadIdx.x; j < wq; j += blockDim.x) {
    float4 v[3][2];
#pragma unroll
    for (int cc = 0; cc < 3; ++cc)
#pragma unroll
      for (int dy = 0; dy < 2; ++dy)
        v[cc][dy] = __ldcs(reinterpret_cast<const float4*>(xr + ((long long)cc * h + dy) * w) + j);
    // Pair k = (dy * 2 + dx) * 3 + cc holds channel k of output pixels 2j
    // (low half, columns 4j + dx) and 2j + 1 (high half, columns 4j + 2 + dx).
    uint32_t out[2][3] = {{0u, 0u, 0u}, {0u, 0u, 0u}};
    bool slow = false;
#pragma unroll
    for (int dy = 0; dy < 2; ++dy)
#pragma unroll
      for (int dx = 0; dx < 2; ++dx)
#pragma unroll
        for (int cc = 0; cc < 3; ++cc) {
          const float4& f = v[cc][dy];
          const int k = (dy * 2 + dx) * 3 + cc;
          const uint64_t t = s2d_mul2(s2d_pair(dx == 0 ? f.x : f.y, dx == 0 ? f.z : f.w), rs2);
          const uint64_t rt = s2d_add2(s2d_add2(t, magic2), nmagic2);
          const uint64_t d = s2d_add2(t, rt ^ 0x8000000080000000ull);  // t - rint(t)
          slow |= fabsf(__uint_as_float(uint32_t(d))) > 0.49975586f;
          slow |= fabsf(__uint_as_float(uint32_t(d >> 32))) > 0.49975586f;
          const float c0 = fminf(fmaxf(__uint_as_float(uint32_t(t)), qnf), qpf);
          const float c1 = fminf(fmaxf(__uint_as_float(uint32_t(t >> 32)), qnf), qpf);
          const uint64_t r = s2d_add2(s2d_pair(c0, c1), magic2);
          out[0][k / 4] |= (uint32_t(r) & 0xFFu) << (8 * (k % 4));
          out[1][k / 4] |= (uint32_t(r >> 32) & 0xFFu) << (8 * (k % 4));
        }
    if (slow) {  // some t within 2^-12 of a half-integer: reload and redo the thread's values exactly
#pragma unroll
      for (int pp = 0; pp < 2; ++pp)
#pragma unroll
        for (int wd = 0; wd < 3; ++wd) out[pp][wd] = 0u;
#pragma unroll
      for (int dy = 0; dy < 2; ++dy)
#pragma unroll
        for (int dx = 0; dx < 2; ++dx)
#pragma unroll
          for (int cc = 0; cc < 3; ++cc) {
            const float4 f = reinterpret_cast<const float4*>(xr + ((long long)cc * h + dy) * w)[j];
            const int k = (dy * 2 + dx) * 3 + cc;
            const int q0 = quant_rs(dx == 0 ? f.x : f.y, scale, rs, qnf, qpf);
            const int q1 = quant_rs(dx == 0 ? f.z : f.w, scale, rs, qnf, qpf);
            out[0][k / 4] |= (uint32_t(q0) & 0xFFu) << (8 * (k % 4));
            out[1][k / 4] |= (uint32_t(q1) & 0xFFu) << (8 * (k % 4));
          }
    }
    uint4* dst = reinterpret_cast<uint4*>(yr + (2 * j) * 16);
    dst[0] = make_uint4(out[0][0], out[0][1], out[0][2], 0u);
    dst[1] = make_uint4(out[1][0], out[1][1], out[1][2], 0u);
  }
}

// Reference explicit lowering: cols[row, c*9 + ky*3 + kx]; out-of-image
// taps quantise 0.0, columns >= c*9 are 0.
__global__ void lower_q3x3_kernel(const float* __restrict__ x, int8_t* __restrict__ cols, int n, int c, int h,
                                  int w, int padded_k, float scale, int qn, int qp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  const long long total = (long long)n * h * w * padded_k;
  const int kpr = c * 9;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / padded_k;
    const int col = int(i - row * padded_k);
    if (col >= kpr) {
      cols[i] = 0;
      continue;
    }
    const int img = int(row / ((long long)h * w));
    const int hw = int(row - (long long)img * h * w);
    const int oh = hw / w, ow = hw % w;
    const int ch = col / 9, k = col % 9;
    const int ih = oh + k / 3 - 1, iw = ow + k % 3 - 1;
    float v = 0.0f;
    if (ih >= 0 && ih < h && iw >= 0 && iw < w) v = x[(((long long)img * c + ch) * h + ih) * w + iw];
    cols[i] = int8_t(quant1(v, scale, qn, qp));
  }
}

__device__ __forceinline__ uint32_t nibble_at(const uint8_t* row, long long k) {
  const uint8_t b = row[k >> 1];
  return (k & 1) ? (b >> 4) : (b & 0xF);
}

// One thread per output byte (two nibbles) of the reordered weights.
__global__ void repack_kernel(const uint8_t* __restrict__ w_in, long long ld_in, int o, int c, int kh, int kw,
                              uint8_t* __restrict__ w_out, long long ld_out, int cp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  const int taps = kh * kw;
  const int cg = cp < 128 ? cp : 128;
  const long long k_out = (long long)taps * cp;
  const long long total = (long long)o * ld_out;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / ld_out;
    const long long byte = i - r * ld_out;
    uint32_t v = 0;
    for (int half = 0; half < 2; ++half) {
      const long long kk = byte * 2 + half;
      if (kk >= k_out) continue;
      const long long g = kk / ((long long)taps * cg);
      const long long rem = kk - g * taps * cg;
      const int t = int(rem / cg);
      const int ch = int(g * cg + rem % cg);
      if (ch < c) v |= nibble_at(w_in + r * ld_in, (long long)ch * taps + t) << (4 * half);
    }
    w_out[i] = uint8_t(v);
  }
}

// NHWC fp32 3x3/s2/p1 max pooling; one thread per (pixel, 4 channels).
__global__ void maxpool_kernel(const float* __restrict__ x, float* __restrict__ yf, int8_t* __restrict__ yq,
                               int n, int h, int w, int c, int ho, int wo, float scale, int qn, int qp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  const int c4 = c / 4;
  const long long total = (long long)n * ho * wo * c4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int cc = int(i % c4) * 4;
    long long t = i / c4;
    const int ow = int(t % wo);
    t /= wo;
    const int oh = int(t % ho);
    const int img = int(t / ho);
    float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int dy = 0; dy < 3; ++dy) {
      const int ih = 2 * oh - 1 + dy;
      if (ih < 0 || ih >= h) continue;
      for (int dx = 0; dx < 3; ++dx) {
        const int iw = 2 * ow - 1 + dx;
        if (iw < 0 || iw >= w) continue;
        const float4 v = *reinterpret_cast<const float4*>(x + (((long long)img * h + ih) * w + iw) * c + cc);
        m[0] = fmaxf(m[0], v.x);
        m[1] = fmaxf(m[1], v.y);
        m[2] = fmaxf(m[2], v.z);
        m[3] = fmaxf(m[3], v.w);
      }
    }
    const long long o = (((long long)img * ho + oh) * wo + ow) * c + cc;
    if (yf) *reinterpret_cast<float4*>(yf + o) = make_float4(m[0], m[1], m[2], m[3]);
    if (yq) {
      uint32_t word = 0;
      for (int j = 0; j < 4; ++j) word |= (uint32_t(quant1(m[j], scale, qn, qp)) & 0xFFu) << (8 * j);
      *reinterpret_cast<uint32_t*>(yq + o) = word;
    }
  }
}

// Mean over hw (sequential float32 sum in (h, w) order, then / hw) + quantise.
__global__ void avgpool_q_kernel(const float* __restrict__ x, int8_t* __restrict__ q, long long ldq, int n, int hw,
                                 int c, float scale, int qn, int qp) {
  w4a8::pdl_trigger();
  w4a8::pdl_wait();
  const long long total = (long long)n * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = int(i % c);
    const int img = int(i / c);
    const float* xi = x + (long long)img * hw * c + ch;
    float s = 0.0f;
    if (hw == 49) {
      // 7 x 7 (the ResNet head), fully unrolled: more loads in flight per
      // thread (12.3 -> 10.0 us at batch 256, 512 channels). The adds keep
      // their order (pixel 0, 1, 2, ...).
      float v[49];
#pragma unroll
      for (int p = 0; p < 49; ++p) v[p] = __ldg(xi + (long long)p * c);
#pragma unroll
      for (int p = 0; p < 49; ++p) s = __fadd_rn(s, v[p]);
    } else {
      // Unrolled so that several pixels' loads are in flight; the adds keep
      // their order (pixel 0, 1, 2, ...).
#pragma unroll 8
      for (int p = 0; p < hw; ++p) s = __fadd_rn(s, __ldg(xi + (long long)p * c));
    }
    const float mean = __fdiv_rn(s, float(hw));
    q[(long long)img * ldq + ch] = int8_t(quant1(mean, scale, qn, qp));
  }
}

int finish() { return cudaGetLastError() == cudaSuccess ? W4A8_OK : W4A8_ERR_LAUNCH; }

// Every helper kernel goes out with programmatic dependent launch, like the
// tensor-core kernels: it starts early and waits (pdl_wait, its first
// statement) for the kernel ahead of it in the stream.
template <typename... Exp, typename... Act>
int launch(void (*kern)(Exp...), dim3 grid, dim3 block, cudaStream_t st, Act&&... args) {
  if (w4a8::launch_kernel(kern, grid, block, 0, st, std::forward<Act>(args)...) != cudaSuccess) return W4A8_ERR_LAUNCH;
  return finish();
}

}  // namespace

extern "C" int w4a8_quantize_rows(const float* x, int64_t ldx, int8_t* q, int64_t ldq, int64_t rows, int cols,
                                  float scale, int qn, int qp, void* stream) {
  if (rows < 0 || cols < 0 || ldx < cols || ldq < cols || !q_ok(scale, qn, qp)) return W4A8_ERR_ARG;
  if (rows == 0 || ldq == 0) return W4A8_OK;
  if (!x || !q) return W4A8_ERR_ARG;
  return launch(quantize_rows_kernel, dim3(grid_for(rows * ldq, 256)), dim3(256), (cudaStream_t)stream,
                x, ldx, q, ldq, rows, cols, scale, qn, qp);
}

extern "C" int w4a8_quantize_nchw_to_nhwc(const float* x, int8_t* y, int n, int c, int h, int w, int c_pad,
                                          float scale, int qn, int qp, void* stream) {
  if (n < 0 || c < 1 || h < 1 || w < 1 || c_pad < c || !q_ok(scale, qn, qp)) return W4A8_ERR_ARG;
  if (n == 0) return W4A8_OK;
  if (!x || !y) return W4A8_ERR_ARG;
  if (n > 65535) return W4A8_ERR_UNSUPPORTED;
  const int hw = h * w;
  dim3 grid((hw + 31) / 32, (c_pad + 31) / 32, n);
  return launch(nchw_to_nhwc_q_kernel, dim3(grid), dim3(32, 8), (cudaStream_t)stream,
                x, y, c, hw, c_pad, scale, qn, qp);
}

extern "C" int w4a8_s2d_quantize(const float* x, int8_t* y, int n, int c, int h, int w, int c_pad, float scale,
                                 int qn, int qp, void* stream) {
  if (n < 0 || c < 1 || h < 2 || w < 2 || (h & 1) || (w & 1) || c_pad < 4 * c || (c_pad % 16) ||
      !q_ok(scale, qn, qp))
    return W4A8_ERR_ARG;
  if (n == 0) return W4A8_OK;
  if (!x || !y) return W4A8_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(y) & 15) return W4A8_ERR_ALIGN;
  const long long total = (long long)n * (h / 2) * (w / 2);
  const long long rows = (long long)n * (h / 2);
  if (c == 3 && c_pad == 16 && w % 4 == 0 && h % 2 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      rows < (1ll << 31) - 4) {
    const float rs = 1.0f / scale;  // IEEE single division on the host: fl(1/s), as the guard band assumes
    const int bx = std::min(w / 4, 128), by = std::max(1, 256 / bx);  // whole rows of column pairs per block
    return launch(s2d_q3_vec_kernel, dim3(unsigned((rows + by - 1) / by)), dim3(bx, by), (cudaStream_t)stream,
                  x, y, n, h, w, scale, rs, qn, qp);
  }
  return launch(s2d_q_kernel, dim3(grid_for(total, 128)), dim3(128), (cudaStream_t)stream,
                x, y, n, c, h, w, c_pad, scale, qn, qp);
}

extern "C" int w4a8_lower_quantize_3x3(const float* x, int8_t* cols, int n, int c, int h, int w, int padded_k,
                                       float scale, int qn, int qp, void* stream) {
  if (n < 0 || c < 0 || h < 0 || w < 0 || padded_k < c * 9 || !q_ok(scale, qn, qp)) return W4A8_ERR_ARG;
  const long long total = (long long)n * h * w * padded_k;
  if (total == 0) return W4A8_OK;
  if (!x || !cols) return W4A8_ERR_ARG;
  return launch(lower_q3x3_kernel, dim3(grid_for(total, 256)), dim3(256), (cudaStream_t)stream,
                x, cols, n, c, h, w, padded_k, scale, qn, qp);
}

extern "C" int w4a8_repack_oihw_int4(const uint8_t* w_in, int64_t ld_in, int o, int c, int kh, int kw,
                                     uint8_t* w_out, int64_t ld_out, int c_pad, void* stream) {
  if (o < 0 || c < 1 || kh < 1 || kw < 1 || c_pad < c || (c_pad > 128 && c_pad % 128)) return W4A8_ERR_ARG;
  const long long k_in = (long long)c * kh * kw, k_out = (long long)c_pad * kh * kw;
  if (ld_in * 2 < k_in || ld_out * 2 < k_out) return W4A8_ERR_ARG;
  if (o == 0) return W4A8_OK;
  if (!w_in || !w_out) return W4A8_ERR_ARG;
  const long long total = (long long)o * ld_out;
  return launch(repack_kernel, dim3(grid_for(total, 256)), dim3(256), (cudaStream_t)stream,
                w_in, ld_in, o, c, kh, kw, w_out, ld_out, c_pad);
}

extern "C" int w4a8_maxpool3x3s2(const float* x_f, float* y_f, int8_t* y_q, int n, int h, int w, int c, int ho,
                                 int wo, float scale, int qn, int qp, void* stream) {
  if (n < 0 || h < 1 || w < 1 || c < 4 || (c % 4) || ho != (h - 1) / 2 + 1 || wo != (w - 1) / 2 + 1)
    return W4A8_ERR_ARG;
  if (y_q && !q_ok(scale, qn, qp)) return W4A8_ERR_ARG;
  if (n == 0) return W4A8_OK;
  if (!x_f || (!y_f && !y_q)) return W4A8_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x_f) & 15) || (reinterpret_cast<uintptr_t>(y_f) & 15) ||
      (reinterpret_cast<uintptr_t>(y_q) & 3))
    return W4A8_ERR_ALIGN;
  const long long total = (long long)n * ho * wo * (c / 4);
  return launch(maxpool_kernel, dim3(grid_for(total, 256)), dim3(256), (cudaStream_t)stream,
                x_f, y_f, y_q, n, h, w, c, ho, wo, scale, qn, qp);
}

extern "C" int w4a8_avgpool_quantize(const float* x, int8_t* q, int64_t ldq, int n, int hw, int c, float scale,
                                     int qn, int qp, void* stream) {
  if (n < 0 || hw < 1 || c < 1 || ldq < c || !q_ok(scale, qn, qp)) return W4A8_ERR_ARG;
  if (n == 0) return W4A8_OK;
  if (!x || !q) return W4A8_ERR_ARG;
  return launch(avgpool_q_kernel, dim3(grid_for((long long)n * c, 256)), dim3(256), (cudaStream_t)stream,
                x, q, ldq, n, hw, c, scale, qn, qp);
}
