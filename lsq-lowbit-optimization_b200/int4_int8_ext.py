"""``int4_int8_ext`` — drop-in for the reference's compiled extension.

The reference builds a pybind11 module of this name from
``csrc/int4_int8_ext.cpp`` (ops registered at :205-212) and imports it by
name in ``quant_pipeline/ops/int4_int8_gemm.py:5-9``. This module keeps the
six op signatures, argument checks and ``RuntimeError`` behaviour of
``csrc/int4_int8_ext.cpp:37-203`` and routes every op to ``libw4a8.so``
(the C ABI declared in ``include/w4a8.h``): tcgen05 int8 MMA kernels for
sm_100a. There is no CPU or eager-torch compute path: without the library
every op raises.

Tensors here only carry device memory; kernels run on the current torch
stream of the input's device, under a device guard.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

import torch

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("W4A8_LIB", _HERE / "libw4a8.so"))

W_INT8, W_INT4 = 0, 1
OUT_S32, OUT_F32, OUT_F16, OUT_S8 = 0, 1, 2, 3
LAYOUT_NHWC, LAYOUT_NCHW = 0, 1

_STATUS = {
    0: "ok",
    1: "invalid argument",
    2: "alignment (pointer or stride not 16-byte aligned)",
    3: "unsupported geometry",
    4: "TMA tensor map rejected",
    -1: "CUDA launch error",
    -2: "device-side wait timeout",
}


class Epilogue(ctypes.Structure):
    """Mirror of ``w4a8_epilogue`` (include/w4a8.h)."""

    _fields_ = [
        ("out_kind", ctypes.c_int),
        ("relu", ctypes.c_int),
        ("alpha", ctypes.c_void_p),
        ("alpha_scalar", ctypes.c_float),
        ("beta", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("res_ld", ctypes.c_int64),
        ("out_scale", ctypes.c_float),
        ("qn", ctypes.c_int),
        ("qp", ctypes.c_int),
        ("aux", ctypes.c_void_p),
        ("aux_ld", ctypes.c_int64),
    ]


class ConvGeom(ctypes.Structure):
    """Mirror of ``w4a8_conv_geom`` (include/w4a8.h)."""

    _fields_ = [
        ("n", ctypes.c_int), ("h", ctypes.c_int), ("w", ctypes.c_int), ("c", ctypes.c_int),
        ("kh", ctypes.c_int), ("kw", ctypes.c_int),
        ("stride", ctypes.c_int),
        ("pad_h", ctypes.c_int), ("pad_w", ctypes.c_int),
        ("ho", ctypes.c_int), ("wo", ctypes.c_int),
        ("o", ctypes.c_int),
        ("out_layout", ctypes.c_int),
        ("ldo", ctypes.c_int64),
        ("pool", ctypes.c_int),
    ]


_vp, _i64, _int, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
_SIGNATURES = {
    "w4a8_gemm": [_vp, _i64, _vp, _i64, _int, _int, _int, _int, ctypes.POINTER(Epilogue), _vp, _i64, _vp],
    "w4a8_gemm_splitk": [_vp, _i64, _vp, _i64, _int, _int, _int, _int, ctypes.POINTER(Epilogue), _vp, _i64, _vp,
                         ctypes.c_size_t, _vp],
    "w4a8_gemm_splitk_workspace": [_int, _int, _int, _int, ctypes.POINTER(ctypes.c_size_t)],
    "w4a8_gemm_splitk_noalloc": [_vp, _i64, _vp, _i64, _int, _int, _int, _int, ctypes.POINTER(Epilogue), _vp, _i64,
                                 _vp],
    "w4a8_conv2d": [_vp, _vp, _int, _i64, ctypes.POINTER(ConvGeom), ctypes.POINTER(Epilogue), _vp, _vp],
    "w4a8_quantize_rows": [_vp, _i64, _vp, _i64, _i64, _int, _f32, _int, _int, _vp],
    "w4a8_quantize_nchw_to_nhwc": [_vp, _vp, _int, _int, _int, _int, _int, _f32, _int, _int, _vp],
    "w4a8_s2d_quantize": [_vp, _vp, _int, _int, _int, _int, _int, _f32, _int, _int, _vp],
    "w4a8_lower_quantize_3x3": [_vp, _vp, _int, _int, _int, _int, _int, _f32, _int, _int, _vp],
    "w4a8_repack_oihw_int4": [_vp, _i64, _int, _int, _int, _int, _vp, _i64, _int, _vp],
    "w4a8_maxpool3x3s2": [_vp, _vp, _vp, _int, _int, _int, _int, _int, _int, _f32, _int, _int, _vp],
    "w4a8_avgpool_quantize": [_vp, _vp, _i64, _int, _int, _int, _f32, _int, _int, _vp],
    "w4a8_device_error": [ctypes.POINTER(ctypes.c_uint)],
    "w4a8_abi_version": [],
    "w4a8_num_sms": [],
}
ABI_VERSION = 2
# w4a8_status (include/w4a8.h)
OK, ERR_ARG, ERR_ALIGN, ERR_UNSUPPORTED, ERR_TENSORMAP, ERR_LAUNCH, ERR_DEVICE = 0, 1, 2, 3, 4, -1, -2
NOALLOC_SCRATCH_BYTES = 4 << 20  # W4A8_NOALLOC_SCRATCH_BYTES (include/w4a8.h)

_lib_handle: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Loads libw4a8.so once; raises RuntimeError when it is missing."""
    global _lib_handle
    if _lib_handle is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"CUDA library {LIB_PATH} is not built. Run: python {_HERE / 'build_native.py'}")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        if handle.w4a8_abi_version() != ABI_VERSION:
            raise RuntimeError("libw4a8.so ABI version mismatch; rebuild it")
        _lib_handle = handle
    return _lib_handle


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: libw4a8 status {rc} ({_STATUS.get(rc, 'unknown')})")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _aligned16(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def _round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def device_error() -> int:
    """Synchronises and returns the recorded device-timeout bits (0 = none)."""
    bits = ctypes.c_uint(0)
    rc = lib().w4a8_device_error(ctypes.byref(bits))
    if rc not in (0, -2):
        _check(rc, "w4a8_device_error")
    return int(bits.value)


def num_sms() -> int:
    return int(lib().w4a8_num_sms())


def make_epilogue(out_kind: int, alpha: Optional[torch.Tensor] = None, alpha_scalar: float = 1.0,
                  beta: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                  res_ld: int = 0, relu: bool = False, out_scale: float = 1.0, qn: int = -128,
                  qp: int = 127, aux: Optional[torch.Tensor] = None, aux_ld: int = 0) -> Epilogue:
    for name, t in (("alpha", alpha), ("beta", beta), ("residual", residual), ("aux", aux)):
        if t is not None and (t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous()):
            raise RuntimeError(f"{name} must be a contiguous float32 CUDA tensor")
    epi = Epilogue(out_kind, int(bool(relu)), _ptr(alpha), float(alpha_scalar), _ptr(beta), _ptr(residual),
                   int(res_ld), float(out_scale), int(qn), int(qp), _ptr(aux), int(aux_ld))
    epi._keep = (alpha, beta, residual, aux)  # the struct holds raw pointers: keep the tensors alive
    return epi


# ---------------------------------------------------------------------------
# Low-level wrappers (device tensors in, caller-provided or new outputs).
# ---------------------------------------------------------------------------
def gemm(a: torch.Tensor, w: torch.Tensor, w_kind: int, k: int, epi: Epilogue, out: torch.Tensor) -> torch.Tensor:
    """out = epilogue(a[:, :k] . w^T). ``a`` int8 [M, lda], ``w`` int8 [N, ldw]
    (w_kind W_INT8) or packed uint8 [N, ldw] (W_INT4); row strides in bytes
    must be multiples of 16. ``out`` is row-major with its own row stride."""
    m, n = a.shape[0], w.shape[0]
    with torch.cuda.device(a.device):
        ws_bytes = splitk_workspace_bytes(m, n, k, w_kind)
        if ws_bytes:
            # Small-M INT4 GEMM: split-K into an int32 workspace from torch's
            # stream-ordered allocator (released back to it after this call).
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a.device)
            rc = lib().w4a8_gemm_splitk(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), w_kind, m, n, k,
                                        ctypes.byref(epi), out.data_ptr(), out.stride(0), ws.data_ptr(), ws_bytes,
                                        _stream(a))
            _check(rc, "w4a8_gemm_splitk")
            return out
        rc = lib().w4a8_gemm(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), w_kind, m, n, k,
                             ctypes.byref(epi), out.data_ptr(), out.stride(0), _stream(a))
    _check(rc, "w4a8_gemm")
    return out


_ws_cache: dict = {}


def splitk_workspace_bytes(m: int, n: int, k: int, w_kind: int) -> int:
    """Workspace bytes of the split-K GEMM for this shape on the current
    device (0 when the shape runs unsplit)."""
    key = (torch.cuda.current_device(), m, n, k, w_kind)
    if key not in _ws_cache:
        nbytes = ctypes.c_size_t(0)
        _check(lib().w4a8_gemm_splitk_workspace(m, n, k, w_kind, ctypes.byref(nbytes)), "w4a8_gemm_splitk_workspace")
        _ws_cache[key] = int(nbytes.value)
    return _ws_cache[key]


def conv2d_nhwc(x: torch.Tensor, w: torch.Tensor, w_kind: int, geom: ConvGeom, epi: Epilogue,
                out: torch.Tensor) -> torch.Tensor:
    """Implicit-GEMM convolution of int8 NHWC ``x`` with weights in the
    library's conv order (see include/w4a8.h); ``geom`` gives the shape."""
    with torch.cuda.device(x.device):
        rc = lib().w4a8_conv2d(x.data_ptr(), w.data_ptr(), w_kind, w.stride(0), ctypes.byref(geom),
                               ctypes.byref(epi), out.data_ptr(), _stream(x))
    _check(rc, "w4a8_conv2d")
    return out


def quantize_rows(x: torch.Tensor, scale: float, qn: int, qp: int, ldq: Optional[int] = None) -> torch.Tensor:
    """fp32 [M, K] -> int8 [M, ldq] LSQ codes, zero-filled columns >= K."""
    m, k = x.shape
    ldq = k if ldq is None else ldq
    q = torch.empty((m, ldq), dtype=torch.int8, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib().w4a8_quantize_rows(x.data_ptr(), x.stride(0), q.data_ptr(), ldq, m, k, float(scale), int(qn),
                                      int(qp), _stream(x))
    _check(rc, "w4a8_quantize_rows")
    return q


def quantize_nchw_to_nhwc(x: torch.Tensor, scale: float, qn: int, qp: int, c_pad: int) -> torch.Tensor:
    n, c, h, w = x.shape
    y = torch.empty((n, h, w, c_pad), dtype=torch.int8, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib().w4a8_quantize_nchw_to_nhwc(x.data_ptr(), y.data_ptr(), n, c, h, w, c_pad, float(scale), int(qn),
                                              int(qp), _stream(x))
    _check(rc, "w4a8_quantize_nchw_to_nhwc")
    return y


def repack_oihw_int4(w_packed: torch.Tensor, c: int, kh: int, kw: int, c_pad: int) -> torch.Tensor:
    """Reference packed weights [O, >= c*kh*kw/2] (OIHW flatten order) ->
    packed [O, ldw] in the conv kernel's (ky, kx, c_pad) order."""
    o = w_packed.shape[0]
    ldw = _round_up(kh * kw * c_pad // 2, 16)
    out = torch.empty((o, ldw), dtype=torch.uint8, device=w_packed.device)
    with torch.cuda.device(w_packed.device):
        rc = lib().w4a8_repack_oihw_int4(w_packed.data_ptr(), w_packed.stride(0), o, c, kh, kw, out.data_ptr(),
                                         ldw, c_pad, _stream(w_packed))
    _check(rc, "w4a8_repack_oihw_int4")
    return out


# int8 weight bytes (O x kh x kw x padded C) above which a 4-bit conv's weights
# cannot stay resident in the conv kernel's shared memory. Streamed 4-bit weights
# would be re-expanded for every output tile, so callers expand them once
# (expand_int4_rows) and pass int8 codes instead: same values, same int32 sums.
CONV_STREAMED_W4_BYTES = 160 * 1024


def expand_int4_rows(packed: torch.Tensor) -> torch.Tensor:
    """Packed int4 rows [O, ldw] (low nibble = even element, two's complement)
    -> int8 codes [O, 2 * ldw], row stride a multiple of 16 when ldw is."""
    p = packed.to(torch.int16)
    lo, hi = p & 0xF, (p >> 4) & 0xF
    lo, hi = lo - ((lo & 8) << 1), hi - ((hi & 8) << 1)
    return torch.stack((lo, hi), dim=-1).reshape(packed.shape[0], -1).to(torch.int8).contiguous()


def conv_channels_padded(c: int, stride: int = 1) -> int:
    """Channel count the conv kernel accepts: 16 (stride 1 only), 32, 64 or
    a multiple of 128 — the halo stores one pixel per 16/32/64/128-byte
    swizzled row."""
    if c <= 16 and stride == 1:
        return 16
    for width in (32, 64):
        if c <= width:
            return width
    return _round_up(c, 128)


# ---------------------------------------------------------------------------
# The six reference ops (csrc/int4_int8_ext.cpp:40-203).
# ---------------------------------------------------------------------------
def _check_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")


def _check_contig(t: torch.Tensor, name: str) -> None:
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_bias(bias: Optional[torch.Tensor], o: int, what: str) -> None:
    if bias is None:
        return
    _require(bias.is_cuda, "bias must be a CUDA tensor")
    _require(bias.is_contiguous(), "bias must be contiguous")
    _require(bias.dim() == 1, "bias must be rank-1 [O]")
    _require(bias.dtype == torch.float32, "bias must be float32")
    _require(bias.size(0) == o, f"bias size must match {what}")


def _padded_operand(t: torch.Tensor, cols: int) -> torch.Tensor:
    """Returns ``t`` or a zero-padded copy with ``cols`` columns whose row
    stride and base satisfy the 16-byte rules of the C ABI."""
    if t.shape[1] == cols and t.stride(0) % 16 == 0 and _aligned16(t):
        return t
    out = torch.zeros((t.shape[0], cols), dtype=t.dtype, device=t.device)
    out[:, : t.shape[1]] = t
    return out


def _combined_scale(a_scale: float, w_scale: float) -> float:
    # float(a_scale * w_scale) evaluated in double (csrc/int4_int8_kernels.cu:345).
    return float(torch.tensor(float(a_scale) * float(w_scale), dtype=torch.float64).to(torch.float32))


def _gemm_s32(a: torch.Tensor, b: torch.Tensor, w_kind: int) -> torch.Tensor:
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty((m, n), dtype=torch.int32, device=a.device)
    if m == 0 or n == 0:
        return c
    if k == 0:
        return c.zero_()
    kp = _round_up(k, 32 if w_kind == W_INT4 else 16)
    a_p = _padded_operand(a, kp)
    b_p = _padded_operand(b, kp // 2 if w_kind == W_INT4 else kp)
    return gemm(a_p, b_p, w_kind, kp, make_epilogue(OUT_S32), c)


def int8_int8_gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """C[M, N] int32 = A[M, K] int8 . B[N, K]^T (csrc/int4_int8_ext.cpp:40-53)."""
    _check_cuda(a, "a"); _check_cuda(b, "b")
    _check_contig(a, "a"); _check_contig(b, "b")
    _require(a.dim() == 2, "A must be rank-2 [M, K]")
    _require(b.dim() == 2, "B must be rank-2 [N, K]")
    _require(a.dtype == torch.int8, "A must be int8")
    _require(b.dtype == torch.int8, "B must be int8")
    _require(a.size(1) == b.size(1), "K dimension mismatch")
    return _gemm_s32(a, b, W_INT8)


def int4_int8_gemm(a: torch.Tensor, b_packed: torch.Tensor) -> torch.Tensor:
    """C[M, N] int32 = A[M, K] int8 . unpack(Bp[N, K/2])^T (csrc/int4_int8_ext.cpp:55-71)."""
    _check_cuda(a, "a"); _check_cuda(b_packed, "b_packed")
    _check_contig(a, "a"); _check_contig(b_packed, "b_packed")
    _require(a.dim() == 2, "A must be rank-2 [M, K]")
    _require(b_packed.dim() == 2, "B packed must be rank-2 [N, K/2]")
    _require(a.dtype == torch.int8, "A must be int8")
    _require(b_packed.dtype == torch.uint8, "B packed must be uint8")
    k = a.size(1)
    _require(k % 2 == 0, "K must be even for int4 packed weights")
    _require(b_packed.size(1) * 2 == k, "Packed B last dim must be K/2")
    return _gemm_s32(a, b_packed, W_INT4)


def lower_quantize_3x3_s1_p1(x: torch.Tensor, scale: float, qn: int, qp: int, padded_k: int) -> torch.Tensor:
    """Explicit 3x3 lowering + quantise (csrc/int4_int8_ext.cpp:73-84)."""
    _check_cuda(x, "x"); _check_contig(x, "x")
    _require(x.dim() == 4, "x must be rank-4 [N, C, H, W]")
    _require(x.dtype == torch.float32, "x must be float32")
    _require(qn >= -128 and qp <= 127, "quant range must fit int8")
    _require(scale > 0.0, "scale must be positive")
    _require(padded_k >= x.size(1) * 9, "padded_k must cover C*3*3")
    n, c, h, w = x.shape
    cols = torch.empty((n * h * w, int(padded_k)), dtype=torch.int8, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib().w4a8_lower_quantize_3x3(x.data_ptr(), cols.data_ptr(), n, c, h, w, int(padded_k),
                                           float(scale), int(qn), int(qp), _stream(x))
    _check(rc, "w4a8_lower_quantize_3x3")
    return cols


def _quantize_conv_input(x: torch.Tensor, scale: float, qn: int, qp: int, c_pad: int,
                         pad: int) -> tuple[torch.Tensor, int]:
    """NCHW fp32 -> NHWC int8 codes for the conv kernel. When the code of
    0.0 is not 0 (0 outside [qn, qp]) the reference's lowering fills
    padding with that code, so the border is materialised explicitly and
    the kernel then runs without padding."""
    xq = quantize_nchw_to_nhwc(x, scale, qn, qp, c_pad)
    if pad == 0 or qn <= 0 <= qp:
        return xq, pad
    zero_code = max(qn, min(qp, 0))
    n, h, w, cp = xq.shape
    xb = torch.full((n, h + 2 * pad, w + 2 * pad, cp), zero_code, dtype=torch.int8, device=x.device)
    xb[:, pad:pad + h, pad:pad + w, :] = xq
    return xb, 0


def conv3x3_int4_int8_s1_p1(x: torch.Tensor, w_packed: torch.Tensor, a_scale: float, w_scale: float, qn: int,
                            qp: int, bias: Optional[torch.Tensor], output_half: bool) -> torch.Tensor:
    """Fused 3x3/s1/p1 conv: quantise + implicit GEMM + dequant/bias, NCHW
    out (csrc/int4_int8_ext.cpp:86-124, csrc/int4_int8_kernels.cu:323-373)."""
    _check_cuda(x, "x"); _check_cuda(w_packed, "w_packed")
    _check_contig(x, "x"); _check_contig(w_packed, "w_packed")
    _require(x.dim() == 4, "x must be rank-4 [N, C, H, W]")
    _require(x.dtype == torch.float32, "x must be float32")
    _require(w_packed.dim() == 2, "w_packed must be rank-2 [O, padded_k/2]")
    _require(w_packed.dtype == torch.uint8, "w_packed must be uint8")
    _require(a_scale > 0.0 and w_scale > 0.0, "scales must be positive")
    _require(qn >= -128 and qp <= 127, "quant range must fit int8")
    o = w_packed.size(0)
    _check_bias(bias, o, "out_channels")
    n, c, h, w = x.shape
    _require(w_packed.size(1) * 2 >= c * 9, "padded_k must cover C*3*3")
    out = torch.empty((n, o, h, w), dtype=torch.float16 if output_half else torch.float32, device=x.device)
    if out.numel() == 0:
        return out
    cp = conv_channels_padded(c)
    xq, pad = _quantize_conv_input(x, a_scale, qn, qp, cp, 1)
    wr = repack_oihw_int4(w_packed, c, 3, 3, cp)
    geom = ConvGeom(n, xq.shape[1], xq.shape[2], cp, 3, 3, 1, pad, pad, h, w, o, LAYOUT_NCHW, 0)
    epi = make_epilogue(OUT_F16 if output_half else OUT_F32, alpha_scalar=_combined_scale(a_scale, w_scale),
                        beta=bias)
    return conv2d_nhwc(xq, wr, W_INT4, geom, epi, out)


def linear_int4_int8(x: torch.Tensor, w_packed: torch.Tensor, a_scale: float, w_scale: float, qn: int, qp: int,
                     bias: Optional[torch.Tensor], output_half: bool) -> torch.Tensor:
    """Fused linear: quantise + W4A8 GEMM + dequant/bias
    (csrc/int4_int8_ext.cpp:126-157, csrc/int4_int8_kernels.cu:375-427)."""
    _check_cuda(x, "x"); _check_cuda(w_packed, "w_packed")
    _check_contig(x, "x"); _check_contig(w_packed, "w_packed")
    _require(x.dim() == 2, "x must be rank-2 [M, K]")
    _require(x.dtype == torch.float32, "x must be float32")
    _require(w_packed.dim() == 2, "w_packed must be rank-2 [O, K/2]")
    _require(w_packed.dtype == torch.uint8, "w_packed must be uint8")
    _require(a_scale > 0.0 and w_scale > 0.0, "scales must be positive")
    _require(qn >= -128 and qp <= 127, "quant range must fit int8")
    _require(x.size(1) == w_packed.size(1) * 2, "input K must match packed weight K")
    o = w_packed.size(0)
    _check_bias(bias, o, "out_features")
    m, k = x.shape
    out = torch.empty((m, o), dtype=torch.float16 if output_half else torch.float32, device=x.device)
    if out.numel() == 0:
        return out
    kp = max(32, _round_up(k, 32))
    xq = quantize_rows(x, a_scale, qn, qp, ldq=kp)
    wp = _padded_operand(w_packed, kp // 2)
    epi = make_epilogue(OUT_F16 if output_half else OUT_F32, alpha_scalar=_combined_scale(a_scale, w_scale),
                        beta=bias)
    return gemm(xq, wp, W_INT4, kp, epi, out)


def conv1x1_int4_int8(x: torch.Tensor, w_packed: torch.Tensor, a_scale: float, w_scale: float, qn: int, qp: int,
                      stride_h: int, stride_w: int, bias: Optional[torch.Tensor],
                      output_half: bool) -> torch.Tensor:
    """Fused strided 1x1 conv, NCHW out (csrc/int4_int8_ext.cpp:159-203,
    csrc/int4_int8_kernels.cu:429-500); Ho = (H-1)/sh + 1."""
    _check_cuda(x, "x"); _check_cuda(w_packed, "w_packed")
    _check_contig(x, "x"); _check_contig(w_packed, "w_packed")
    _require(x.dim() == 4, "x must be rank-4 [N, C, H, W]")
    _require(x.dtype == torch.float32, "x must be float32")
    _require(w_packed.dim() == 2, "w_packed must be rank-2 [O, C/2]")
    _require(w_packed.dtype == torch.uint8, "w_packed must be uint8")
    _require(a_scale > 0.0 and w_scale > 0.0, "scales must be positive")
    _require(qn >= -128 and qp <= 127, "quant range must fit int8")
    _require(x.size(1) == w_packed.size(1) * 2, "input C must match packed weight K")
    _require(stride_h >= 1 and stride_w >= 1, "stride must be positive")
    o = w_packed.size(0)
    _check_bias(bias, o, "out_channels")
    n, c, h, w = x.shape
    _require(h >= 1 and w >= 1, "spatial dims must be positive")
    ho, wo = (h - 1) // stride_h + 1, (w - 1) // stride_w + 1
    out = torch.empty((n, o, ho, wo), dtype=torch.float16 if output_half else torch.float32, device=x.device)
    if out.numel() == 0:
        return out
    if stride_h == stride_w and stride_h in (1, 2):
        stride = stride_h
    else:
        stride = 1
    cp = conv_channels_padded(c, stride)
    xq = quantize_nchw_to_nhwc(x, a_scale, qn, qp, cp)
    if not (stride_h == stride_w and stride_h in (1, 2)):
        xq = xq[:, ::stride_h, ::stride_w, :].contiguous()
    wr = repack_oihw_int4(w_packed, c, 1, 1, cp)
    geom = ConvGeom(n, xq.shape[1], xq.shape[2], cp, 1, 1, stride, 0, 0, ho, wo, o, LAYOUT_NCHW, 0)  # noqa: E501
    epi = make_epilogue(OUT_F16 if output_half else OUT_F32, alpha_scalar=_combined_scale(a_scale, w_scale),
                        beta=bias)
    return conv2d_nhwc(xq, wr, W_INT4, geom, epi, out)


def conv_nchw(x: torch.Tensor, w_conv: torch.Tensor, w_kind: int, c: int, kh: int, kw: int, stride: int, pad: int,
              a_scale: float, qn: int, qp: int, alpha_scalar: float = 1.0, alpha: Optional[torch.Tensor] = None,
              bias: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
              pad_code_of_zero: bool = False) -> torch.Tensor:
    """fp32 NCHW conv through the implicit-GEMM kernel, NCHW out.

    ``w_conv`` holds weights already in the kernel's conv order (see
    repack_oihw_int4). ``pad_code_of_zero`` selects the fused 3x3 op's
    padding semantics (padding quantises 0.0) instead of the unfold path's
    (padding is the code 0); the two differ only when 0 is outside [qn, qp].
    """
    n, cx, h, w = x.shape
    o = w_conv.shape[0]
    ho = (h + 2 * pad - kh) // stride + 1
    wo = (w + 2 * pad - kw) // stride + 1
    out = torch.empty((n, o, ho, wo), dtype=out_dtype, device=x.device)
    if out.numel() == 0:
        return out
    cp = conv_channels_padded(c, stride)
    if pad_code_of_zero:
        xq, p = _quantize_conv_input(x, a_scale, qn, qp, cp, pad)
    else:
        xq, p = quantize_nchw_to_nhwc(x, a_scale, qn, qp, cp), pad
    geom = ConvGeom(n, xq.shape[1], xq.shape[2], cp, kh, kw, stride, p, p, ho, wo, o, LAYOUT_NCHW, 0)
    kind = {torch.float32: OUT_F32, torch.float16: OUT_F16}[out_dtype]
    epi = make_epilogue(kind, alpha=alpha, alpha_scalar=alpha_scalar, beta=bias)
    return conv2d_nhwc(xq, w_conv, w_kind, geom, epi, out)
