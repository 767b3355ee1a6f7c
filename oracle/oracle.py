"""CPU oracle for the W4A8 path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the integer semantics of
peihengzju/lsq-lowbit-optimization. Only ``tests/``, ``__graft_entry__.smoke``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may
import it, and only as the checker or the timed CPU baseline; the product
path (``int4_int8_ext`` -> ``libw4a8.so``) never calls it.

Pinning: the nibble layout, weight padding/packing of the converted modules,
the LSQ adapter conversion and the reference's unfold conv path are checked
against golden vectors produced by the reference's own Python code
(``tests/golden/make_golden.py``); GEMMs follow the reference's own known-
answer check (benchmarks/benchmark_inference.py:62-79).

Conventions (all restated from the reference):
  quantise  q = clamp(rint(x / s), qn, qp), float32 IEEE division and
            round-half-to-even (quant_pipeline/integration/lsq_adapter.py:103-104,
            quant_pipeline/ops/int4_conv2d.py:172, csrc/int4_int8_kernels.cu:162-164)
  GEMM      C = A . B^T with int32 accumulation (csrc/int4_int8_kernels.cu:19-84)
  epilogue  y = float32(acc) * float32(s_a * s_w) + bias, each op rounded
            (csrc/int4_int8_kernels.cu:109-112, :345; int4_conv2d.py:192-195)
Integer products are evaluated with float64 BLAS, exact because every
partial sum is an integer far below 2**53.
"""
from __future__ import annotations

import numpy as np

# ------------------------------------------------------------------ packing
def pack_int4(w: np.ndarray) -> np.ndarray:
    """quant_pipeline/quantization/int4_pack.py:9-27: element 2j -> low
    nibble, 2j+1 -> high nibble of byte j, two's complement, last dim."""
    w = np.asarray(w)
    if w.shape[-1] % 2:
        raise ValueError("Last dimension K must be even for int4 packing")
    if np.any(w < -8) or np.any(w > 7):
        raise ValueError("INT4 tensor contains values outside [-8, 7]")
    lo = (w[..., 0::2].astype(np.int16) & 0xF).astype(np.uint8)
    hi = (w[..., 1::2].astype(np.int16) & 0xF).astype(np.uint8)
    return (lo | (hi << 4)).astype(np.uint8)


def unpack_int4(p: np.ndarray) -> np.ndarray:
    """quant_pipeline/quantization/int4_pack.py:30-50 (sign extension
    (x << 4) >> 4)."""
    p = np.asarray(p, dtype=np.uint8)
    lo = ((p & 0xF).astype(np.int8) << 4) >> 4
    hi = (((p >> 4) & 0xF).astype(np.int8) << 4) >> 4
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


# ------------------------------------------------------------- quantisation
def quantize(x: np.ndarray, scale: float, qn: int, qp: int) -> np.ndarray:
    """clamp(round(x / s), qn, qp) in float32 (lsq_adapter.py:103-104)."""
    x = np.asarray(x, dtype=np.float32)
    q = np.rint(x / np.float32(scale))
    return np.clip(q, qn, qp).astype(np.int8)


def combined_scale(a_scale: float, w_scale: float) -> np.float32:
    """(float)(double(a) * double(w)) (csrc/int4_int8_kernels.cu:345)."""
    return np.float32(np.float64(a_scale) * np.float64(w_scale))


# ------------------------------------------------------------------- GEMMs
def gemm_s32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """A[M,K] . B[N,K]^T with int32 result (benchmarks/benchmark_inference.py:67-76)."""
    a64 = np.asarray(a, dtype=np.float64)
    b64 = np.asarray(b, dtype=np.float64)
    return np.rint(a64 @ b64.T).astype(np.int64).astype(np.int32)


def int4_int8_gemm(a: np.ndarray, b_packed: np.ndarray) -> np.ndarray:
    """int4_int8_gemm (csrc/int4_int8_ext.cpp:55-71): unpack then GEMM."""
    return gemm_s32(a, unpack_int4(b_packed))


def epilogue(acc: np.ndarray, alpha, beta=None, residual=None, relu: bool = False) -> np.ndarray:
    """y = f32(acc)*alpha (+beta) (+residual) (relu), each step rounded to
    float32 (the library's documented epilogue order; the reference's is the
    first two steps, csrc/int4_int8_kernels.cu:109-112)."""
    y = np.asarray(acc).astype(np.float32) * np.asarray(alpha, dtype=np.float32)
    y = y.astype(np.float32)
    if beta is not None:
        y = (y + np.asarray(beta, dtype=np.float32)).astype(np.float32)
    if residual is not None:
        y = (y + np.asarray(residual, dtype=np.float32)).astype(np.float32)
    if relu:
        y = np.maximum(y, np.float32(0.0))
    return y


# ------------------------------------------------------ reference-API ops
def lower_quantize_3x3(x: np.ndarray, scale: float, qn: int, qp: int, padded_k: int) -> np.ndarray:
    """csrc/int4_int8_kernels.cu:202-251: cols[n*h*w, padded_k], column
    c*9 + ky*3 + kx; out-of-image taps quantise 0.0; columns >= c*9 are 0."""
    n, c, h, w = x.shape
    xp = np.zeros((n, c, h + 2, w + 2), dtype=np.float32)
    xp[:, :, 1:h + 1, 1:w + 1] = x
    q = quantize(xp, scale, qn, qp)
    cols = np.zeros((n, h, w, padded_k), dtype=np.int8)
    for ky in range(3):
        for kx in range(3):
            patch = q[:, :, ky:ky + h, kx:kx + w]  # [n, c, h, w]
            cols[..., np.arange(c) * 9 + ky * 3 + kx] = patch.transpose(0, 2, 3, 1)
    return cols.reshape(n * h * w, padded_k)


def unfold_nchw(q: np.ndarray, kh: int, kw: int, stride: int, pad: int) -> np.ndarray:
    """F.unfold-style lowering of an integer NCHW tensor, zero padding,
    K order c*kh*kw + ky*kw + kx (quant_pipeline/ops/int4_conv2d.py:174-181).
    Returns [n*ho*wo, c*kh*kw]."""
    n, c, h, w = q.shape
    ho = (h + 2 * pad - kh) // stride + 1
    wo = (w + 2 * pad - kw) // stride + 1
    qp_ = np.zeros((n, c, h + 2 * pad, w + 2 * pad), dtype=q.dtype)
    qp_[:, :, pad:pad + h, pad:pad + w] = q
    cols = np.empty((n, ho, wo, c, kh, kw), dtype=q.dtype)
    for ky in range(kh):
        for kx in range(kw):
            cols[..., ky, kx] = qp_[:, :, ky:ky + stride * ho:stride, kx:kx + stride * wo:stride].transpose(0, 2, 3, 1)
    return cols.reshape(n * ho * wo, c * kh * kw), ho, wo


def conv3x3_s1_p1(x, w_packed, a_scale, w_scale, qn, qp, bias=None, output_half=False) -> np.ndarray:
    """conv3x3_int4_int8_s1_p1 (csrc/int4_int8_kernels.cu:323-373)."""
    n, c, h, w = x.shape
    padded_k = w_packed.shape[1] * 2
    cols = lower_quantize_3x3(x, a_scale, qn, qp, padded_k)
    acc = int4_int8_gemm(cols, w_packed)  # [n*h*w, o]
    y = epilogue(acc, combined_scale(a_scale, w_scale), bias)
    y = y.reshape(n, h, w, -1).transpose(0, 3, 1, 2)
    return y.astype(np.float16) if output_half else np.ascontiguousarray(y)


def linear(x, w_packed, a_scale, w_scale, qn, qp, bias=None, output_half=False) -> np.ndarray:
    """linear_int4_int8 (csrc/int4_int8_kernels.cu:375-427)."""
    acc = int4_int8_gemm(quantize(x, a_scale, qn, qp), w_packed)
    y = epilogue(acc, combined_scale(a_scale, w_scale), bias)
    return y.astype(np.float16) if output_half else y


def conv1x1(x, w_packed, a_scale, w_scale, qn, qp, stride_h, stride_w, bias=None, output_half=False):
    """conv1x1_int4_int8 (csrc/int4_int8_kernels.cu:429-500): strided
    gather, Ho = (H-1)/sh + 1."""
    n, c, h, w = x.shape
    xs = x[:, :, ::stride_h, ::stride_w]
    ho, wo = xs.shape[2], xs.shape[3]
    cols = quantize(xs, a_scale, qn, qp).transpose(0, 2, 3, 1).reshape(n * ho * wo, c)
    acc = int4_int8_gemm(cols, w_packed)
    y = epilogue(acc, combined_scale(a_scale, w_scale), bias).reshape(n, ho, wo, -1).transpose(0, 3, 1, 2)
    return y.astype(np.float16) if output_half else np.ascontiguousarray(y)


def buffer_scale(a_scale: float, w_scale: float) -> np.float32:
    """a_scale * w_scale of the modules' float32 buffers, multiplied in
    float32 (quant_pipeline/ops/int4_conv2d.py:192). Equal to
    combined_scale whenever both scales are float32 values (as produced by
    the adapter, lsq_adapter.py:124-125)."""
    return np.float32(np.float32(a_scale) * np.float32(w_scale))


def conv_unfold_path(x, w_int, a_scale, w_scale, qn, qp, stride, pad, bias=None, out_dtype=np.float32):
    """The module's general path (quant_pipeline/ops/int4_conv2d.py:171-201):
    quantise, unfold, GEMM, y = acc * (s_a*s_w) + bias with the float32
    buffer product, NCHW."""
    n = x.shape[0]
    o, c, kh, kw = w_int.shape
    q = quantize(x, a_scale, qn, qp)
    cols, ho, wo = unfold_nchw(q, kh, kw, stride, pad)
    acc = gemm_s32(cols, w_int.reshape(o, -1))
    y = epilogue(acc, buffer_scale(a_scale, w_scale), bias)
    return np.ascontiguousarray(y.reshape(n, ho, wo, o).transpose(0, 3, 1, 2)).astype(out_dtype)


# ----------------------------------------------------------- NHWC int8 path
def _exact_float_type(k: int, amax: int, wmax: int):
    """Float type whose BLAS product of integer operands is exact: every
    partial sum is an integer of magnitude <= k * amax * wmax, exact in
    float32 below 2**24 (in any summation order) and in float64 below 2**53."""
    return np.float32 if k * amax * wmax < (1 << 24) else np.float64


def conv_nhwc_s32(xq: np.ndarray, w_ohwi: np.ndarray, stride: int, pad_h: int, pad_w: int, ho: int,
                  wo: int, chunk_bytes: int = 1 << 28) -> np.ndarray:
    """Integer conv of NHWC codes with OHWI weights; zero padding top/left
    pad_h/pad_w, output [n, ho, wo, o] int32. Images are lowered a few at a
    time so that the lowered columns stay below ``chunk_bytes``."""
    n, h, w, c = xq.shape
    o, kh, kw, _ = w_ohwi.shape
    hp = max(h + pad_h, (ho - 1) * stride + kh)
    wp = max(w + pad_w, (wo - 1) * stride + kw)
    k = kh * kw * c
    amax = int(np.abs(xq.astype(np.int32)).max()) if xq.size else 0
    wmax = int(np.abs(w_ohwi.astype(np.int32)).max()) if w_ohwi.size else 0
    ft = _exact_float_type(k, amax, wmax)
    wt = np.ascontiguousarray(w_ohwi.reshape(o, -1).astype(ft).T)
    out = np.empty((n, ho, wo, o), dtype=np.int32)
    per_img = ho * wo * k * np.dtype(ft).itemsize
    step = max(1, int(chunk_bytes // max(per_img, 1)))
    for i0 in range(0, n, step):
        i1 = min(n, i0 + step)
        xp = np.zeros((i1 - i0, hp, wp, c), dtype=ft)
        xp[:, pad_h:pad_h + h, pad_w:pad_w + w, :] = xq[i0:i1]
        cols = np.empty((i1 - i0, ho, wo, kh, kw, c), dtype=ft)
        for ky in range(kh):
            for kx in range(kw):
                cols[:, :, :, ky, kx, :] = xp[:, ky:ky + stride * ho:stride, kx:kx + stride * wo:stride, :]
        acc = cols.reshape(-1, k) @ wt
        out[i0:i1] = np.rint(acc).astype(np.int64).astype(np.int32).reshape(i1 - i0, ho, wo, o)
    return out


def maxpool3x3s2(x: np.ndarray) -> np.ndarray:
    """3x3/s2/p1 max pooling of NHWC float32, padding never selected."""
    n, h, w, c = x.shape
    ho, wo = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    xp = np.full((n, h + 2, w + 2, c), -np.inf, dtype=np.float32)
    xp[:, 1:h + 1, 1:w + 1] = x
    out = np.full((n, ho, wo, c), -np.inf, dtype=np.float32)
    for dy in range(3):
        for dx in range(3):
            out = np.maximum(out, xp[:, dy:dy + 2 * ho:2, dx:dx + 2 * wo:2])
    return out


def avgpool(x: np.ndarray) -> np.ndarray:
    """Mean over (h, w) of NHWC float32: sequential float32 sum in (h, w)
    order, then divided by h*w."""
    n, h, w, c = x.shape
    s = np.cumsum(x.reshape(n, h * w, c), axis=1, dtype=np.float32)[:, -1, :]
    return (s / np.float32(h * w)).astype(np.float32)
