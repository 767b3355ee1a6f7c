/*
 * libw4a8 — C ABI of the B200 (sm_100a) W4A8 inference path.
 *
 * Plain C: device pointers, sizes in elements unless noted, a CUDA stream as
 * an opaque pointer (NULL = legacy default stream), an int status return.
 * Nothing here allocates device memory; callers own every buffer. All calls
 * are asynchronous with respect to the host (kernels are enqueued on
 * `stream`), except w4a8_device_error which synchronises the device.
 * Kernels are launched with programmatic dependent launch: one may start
 * while the kernel ahead of it in `stream` finishes, and it waits for that
 * kernel to complete before it reads or writes global memory, so stream
 * order holds. W4A8_PDL=0 in the environment launches in plain stream order.
 *
 * Reference interfaces replaced (peihengzju/lsq-lowbit-optimization):
 *   csrc/int4_int8_ext.cpp:205-212   the six pybind ops of `int4_int8_ext`
 *   csrc/int4_int8_kernels.cu:257-500 their host launchers
 * The Python module `int4_int8_ext` in this repository binds these symbols
 * with ctypes and keeps the six reference signatures.
 */
#ifndef W4A8_H_
#define W4A8_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define W4A8_API __attribute__((visibility("default")))
#else
#define W4A8_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define W4A8_ABI_VERSION 2

/* Status codes: 0 ok, > 0 argument errors (nothing was launched),
 * < 0 runtime errors. */
enum {
  W4A8_OK = 0,
  W4A8_ERR_ARG = 1,         /* bad shape, range or null pointer           */
  W4A8_ERR_ALIGN = 2,       /* pointer or stride violates 16-byte rules    */
  W4A8_ERR_UNSUPPORTED = 3, /* geometry outside what the kernels handle    */
  W4A8_ERR_TENSORMAP = 4,   /* cuTensorMapEncodeTiled rejected a map       */
  W4A8_ERR_LAUNCH = -1,     /* cudaLaunch / attribute error                */
  W4A8_ERR_DEVICE = -2      /* a kernel recorded a bounded-wait timeout    */
};

/* Weight operand encodings. */
enum {
  W4A8_W_INT8 = 0,  /* int8 [N, ldw]                                      */
  W4A8_W_INT4 = 1   /* packed int4 [N, ldw] bytes, int4_pack nibble layout:
                       byte j = (w[2j] & 0xF) | (w[2j+1] & 0xF) << 4       */
};

/* Output element kinds. */
enum {
  W4A8_OUT_S32 = 0, /* raw int32 accumulator                                */
  W4A8_OUT_F32 = 1,
  W4A8_OUT_F16 = 2, /* round-to-nearest-even                                */
  W4A8_OUT_S8 = 3   /* requantised LSQ codes                                */
};

/* Output layouts of the convolution. */
enum { W4A8_LAYOUT_NHWC = 0, W4A8_LAYOUT_NCHW = 1 };

/*
 * Fused epilogue, applied per output element (row r, column n) in this
 * exact float32 order (each step rounded to nearest even, no contraction):
 *   y = float(acc) * alpha[n]         (alpha_scalar when alpha == NULL)
 *   y = y + beta[n]                   (skipped when beta == NULL)
 *   y = y + residual[r * res_ld + n]  (skipped when residual == NULL)
 *   y = max(y, 0)                     (when relu != 0)
 *   aux[r * aux_ld + n] = y           (when aux != NULL)
 *   out = y, or for W4A8_OUT_S8: clamp(rint(y / out_scale), qn, qp)
 * For W4A8_OUT_S32 the raw accumulator is stored and the rest is ignored.
 */
typedef struct {
  int out_kind;
  int relu;
  const float* alpha;
  float alpha_scalar;
  const float* beta;
  const float* residual;
  int64_t res_ld;
  float out_scale;
  int qn;
  int qp;
  float* aux;
  int64_t aux_ld;
} w4a8_epilogue;

/*
 * C[M, N] = epilogue( A[M, K] . W[N, K]^T ), int32 accumulation on the
 * tcgen05 tensor cores.
 *   A   int8, row stride lda bytes.
 *   W   w_kind encoding, row stride ldw bytes (K/2 payload bytes for INT4).
 *   C   row stride ldc elements of the output kind.
 * Rules: lda, ldw multiples of 16; A, W 16-byte aligned; K even for INT4.
 * Replaces int8_int8_gemm / int4_int8_gemm (csrc/int4_int8_ext.cpp:40-71,
 * csrc/int4_int8_kernels.cu:257-291) and the GEMM+epilogue of
 * linear_int4_int8 (csrc/int4_int8_kernels.cu:375-427).
 */
W4A8_API int w4a8_gemm(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int w_kind, int M, int N, int K,
              const w4a8_epilogue* epi, void* C, int64_t ldc, void* stream);

/*
 * Split-K form of w4a8_gemm for INT4 weights whose output tiles alone cannot
 * fill the GPU (small M: decode-style linear layers). The k-blocks are split
 * into ranges whose int32 partial sums are added (exactly) into `workspace`
 * (int32 [M, N], zeroed by the call), then the epilogue runs over the sums.
 * Results are identical to w4a8_gemm. workspace_bytes must be at least what
 * w4a8_gemm_splitk_workspace reports; with a null workspace, INT8 weights
 * or a shape that needs no split this is w4a8_gemm. Calls sharing one
 * workspace must be ordered (one stream).
 * Extends the reference's int4_int8_gemm path (csrc/int4_int8_kernels.cu:257-291),
 * which has no split-K.
 */
W4A8_API int w4a8_gemm_splitk(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int w_kind, int M, int N,
                              int K, const w4a8_epilogue* epi, void* C, int64_t ldc, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Workspace bytes w4a8_gemm_splitk needs for this shape (0: no split). */
W4A8_API int w4a8_gemm_splitk_workspace(int M, int N, int K, int w_kind, size_t* bytes);

/*
 * w4a8_gemm_splitk for callers that cannot allocate device memory. Examples
 * are plugins and serving runtimes whose device memory belongs to the host
 * application's own pool or fixed budget: there a cudaMalloc can fail or
 * break the budget, and cudaMalloc / cudaFree synchronise the whole device,
 * stalling every other stream. This entry point needs no workspace. The
 * caller passes only inputs and outputs, and the int32 split-K partial sums
 * go to one fixed array of W4A8_NOALLOC_SCRATCH_BYTES (4 MiB) inside the
 * library. Every GPU that loads the library holds that array until the
 * process exits.
 * - INT4 weights only. Shapes that take no split (few-token GEMV, or
 *   enough output tiles to fill the GPU) never touch the array and run as
 *   w4a8_gemm at any size. Split-K shapes with M * N * 4 above
 *   W4A8_NOALLOC_SCRATCH_BYTES are rejected with W4A8_ERR_ARG and nothing
 *   is launched (w4a8_gemm_splitk_workspace reports whether a shape splits).
 * - Results equal w4a8_gemm.
 * - The first call on a device looks up the array's device address (once per
 *   device, with that device current). Make that first call before any
 *   stream capture.
 * - Each call clears the part of the array it uses.
 * - All calls on a device share the one array, so calls that overlap on the
 *   GPU (different streams, or several host threads) race and corrupt each
 *   other's results. Order them on one stream.
 * No counterpart in the reference.
 */
#define W4A8_NOALLOC_SCRATCH_BYTES (4u << 20)
W4A8_API int w4a8_gemm_splitk_noalloc(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int w_kind, int M,
                                      int N, int K, const w4a8_epilogue* epi, void* C, int64_t ldc, void* stream);

/* Convolution geometry. Input is int8 NHWC [n, h, w, c] with c in
 * {16, 32, 64} or c a multiple of 128 (pad channels with zero codes and
 * zero weights otherwise); c == 16 only at stride 1.
 * Weights are [o, groups, kh*kw, c/groups_of_128] in the w_kind encoding:
 * for c <= 128 that is OHWI ([o][kh][kw][c]); for c > 128 channels are
 * split in groups of 128 and the group index is outermost. Row stride ldw
 * bytes (multiple of 16). Padding rows/columns read zero codes. */
typedef struct {
  int n, h, w, c;
  int kh, kw;
  int stride;        /* 1 or 2 */
  int pad_h, pad_w;  /* top / left zero padding */
  int ho, wo;        /* output size (bottom / right padding implied) */
  int o;             /* output channels */
  int out_layout;    /* W4A8_LAYOUT_NHWC or W4A8_LAYOUT_NCHW */
  int64_t ldo;       /* NHWC: output elements per pixel (>= o) */
  int pool;          /* 1: fuse a 3x3/s2/p1 max pool after the epilogue
                        (8-bit weights, o <= 64, NHWC out); outputs are then pooled, of size
                        ((ho-1)/2+1, (wo-1)/2+1). 0: no pooling. */
} w4a8_conv_geom;

/*
 * Implicit-GEMM convolution: out = epilogue(conv(x, W)); rows of the GEMM
 * are output pixels (n, oh, ow), columns output channels. residual / aux of
 * the epilogue are NHWC fp32 with res_ld / aux_ld elements per pixel.
 * With geom->pool the 3x3/s2/p1 max pool is taken over the int32
 * accumulators before the epilogue (exact: the epilogue is monotone in the
 * accumulator, increasing where alpha >= 0 and decreasing where alpha < 0,
 * so the extreme accumulator of each window yields the pooled value);
 * residual is not allowed then.
 * Replaces the lowering + GEMM + postprocess chain of
 * conv3x3_int4_int8_s1_p1 and conv1x1_int4_int8
 * (csrc/int4_int8_kernels.cu:323-373, 429-500).
 */
W4A8_API int w4a8_conv2d(const int8_t* x, const void* W, int w_kind, int64_t ldw, const w4a8_conv_geom* g,
                const w4a8_epilogue* epi, void* out, void* stream);

/* q[r, k] = clamp(rint(x[r, k] / scale), qn, qp) for k < cols and 0 for
 * cols <= k < ldq. x row stride ldx elements. (quantize_2d_kernel,
 * csrc/int4_int8_kernels.cu:149-165, with IEEE division.) */
W4A8_API int w4a8_quantize_rows(const float* x, int64_t ldx, int8_t* q, int64_t ldq, int64_t rows, int cols, float scale,
                       int qn, int qp, void* stream);

/* NCHW float32 [n, c, h, w] -> NHWC int8 [n, h, w, c_pad] LSQ codes,
 * channels >= c written as 0. */
W4A8_API int w4a8_quantize_nchw_to_nhwc(const float* x, int8_t* y, int n, int c, int h, int w, int c_pad, float scale,
                               int qn, int qp, void* stream);

/* Space-to-depth by 2 fused with quantisation for the 7x7/s2 stem:
 * y[n, Y, X, (dy*2+dx)*c + ch] = q(x[n, ch, 2Y+dy, 2X+dx]), channels
 * >= 4c zero up to c_pad. h and w even. */
W4A8_API int w4a8_s2d_quantize(const float* x, int8_t* y, int n, int c, int h, int w, int c_pad, float scale, int qn,
                      int qp, void* stream);

/* Reference op lower_quantize_3x3_s1_p1 (csrc/int4_int8_kernels.cu:202-251):
 * cols[n*h*w, padded_k] int8, column c*9+ky*3+kx, padding and columns
 * >= c*9 quantised from 0.0 / set to 0 exactly as the reference does. */
W4A8_API int w4a8_lower_quantize_3x3(const float* x, int8_t* cols, int n, int c, int h, int w, int padded_k, float scale,
                            int qn, int qp, void* stream);

/* Reorders packed int4 weights from the reference's OIHW flatten order
 * (k = c*kh*kw + ky*kw + kx, ld_in bytes per row) to this library's conv
 * order (ky, kx, c) with c padded to c_pad (zero nibbles), channel groups
 * of 128 outermost when c_pad > 128; ld_out bytes per output row. */
W4A8_API int w4a8_repack_oihw_int4(const uint8_t* w_in, int64_t ld_in, int o, int c, int kh, int kw, uint8_t* w_out,
                          int64_t ld_out, int c_pad, void* stream);

/* 3x3 stride-2 pad-1 max pooling of an NHWC fp32 tensor [n, h, w, c]
 * (padding never wins, as with -inf padding). Writes y_f [n, ho, wo, c]
 * when non-NULL and the LSQ codes y_q = clamp(rint(max / scale), qn, qp)
 * when non-NULL (quantisation is monotone, so this equals pooling the
 * codes). c % 4 == 0. */
W4A8_API int w4a8_maxpool3x3s2(const float* x_f, float* y_f, int8_t* y_q, int n, int h, int w, int c, int ho, int wo,
                      float scale, int qn, int qp, void* stream);

/* Global average pooling of an NHWC fp32 tensor followed by quantisation:
 * q[n, c] = clamp(rint(mean_hw(x) / scale), qn, qp); mean is summed in
 * (h, w) order in float32 and divided by h*w. */
W4A8_API int w4a8_avgpool_quantize(const float* x, int8_t* q, int64_t ldq, int n, int hw, int c, float scale, int qn,
                          int qp, void* stream);

/* Synchronises the current device, then returns W4A8_ERR_DEVICE and the
 * recorded bits in *bits if any kernel of this library gave up on a wait
 * since the last call (the word is cleared), else W4A8_OK. */
W4A8_API int w4a8_device_error(unsigned* bits);

/* ABI version (W4A8_ABI_VERSION) and the number of SMs the tile
 * schedulers size persistent grids for on the current device. */
W4A8_API int w4a8_abi_version(void);
W4A8_API int w4a8_num_sms(void);

#ifdef __cplusplus
}
#endif

#endif /* W4A8_H_ */
