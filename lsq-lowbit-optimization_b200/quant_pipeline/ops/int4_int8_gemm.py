"""Python op wrappers over ``int4_int8_ext`` — same six functions, argument
casting and ``RuntimeError`` when the native library is absent as
quant_pipeline/ops/int4_int8_gemm.py:1-153 of the reference."""
import torch

from quant_pipeline.quantization.int4_pack import pack_int4_weights

try:
    import int4_int8_ext
    int4_int8_ext.lib()
    _import_error = None
except (ImportError, RuntimeError, OSError) as exc:  # library missing or unloadable
    int4_int8_ext = None
    _import_error = exc


def _check_ext_loaded() -> None:
    if int4_int8_ext is None:
        raise RuntimeError(
            "CUDA extension int4_int8_ext is not built. "
            "Run: python lsq-lowbit-optimization_b200/build_native.py"
        ) from _import_error


def int8_int8_gemm(a_int8: torch.Tensor, b_int8: torch.Tensor) -> torch.Tensor:
    """C[M, N] int32 = A[M, K] int8 @ B[N, K]^T int8 (CUDA, contiguous)."""
    _check_ext_loaded()
    return int4_int8_ext.int8_int8_gemm(a_int8, b_int8)


def int4_int8_gemm(a_int8: torch.Tensor, b_int4_or_packed: torch.Tensor) -> torch.Tensor:
    """INT4-storage / INT8-compute GEMM; B is either [N, K] int8 values in
    [-8, 7] (packed on the fly) or [N, K/2] uint8 already packed."""
    _check_ext_loaded()
    if b_int4_or_packed.dtype == torch.uint8:
        b_packed = b_int4_or_packed
    else:
        b_packed = pack_int4_weights(b_int4_or_packed)
    return int4_int8_ext.int4_int8_gemm(a_int8, b_packed)


def lower_quantize_3x3_s1_p1(x_fp32: torch.Tensor, scale: float, qn: int, qp: int, padded_k: int) -> torch.Tensor:
    """Quantise + explicit 3x3/s1/p1 lowering: [N, C, H, W] f32 -> [N*H*W, padded_k] int8."""
    _check_ext_loaded()
    return int4_int8_ext.lower_quantize_3x3_s1_p1(x_fp32, float(scale), int(qn), int(qp), int(padded_k))


def conv3x3_int4_int8_s1_p1(x_fp32, w_packed, a_scale, w_scale, qn, qp, bias=None, out_dtype=torch.float16):
    """Fused 3x3/s1/p1 convolution (quantise + implicit GEMM + dequant/bias), NCHW out."""
    _check_ext_loaded()
    return int4_int8_ext.conv3x3_int4_int8_s1_p1(x_fp32, w_packed, float(a_scale), float(w_scale), int(qn),
                                                 int(qp), bias, bool(out_dtype == torch.float16))


def linear_int4_int8(x_fp32, w_packed, a_scale, w_scale, qn, qp, bias=None, out_dtype=torch.float16):
    """Fused W4A8 linear (quantise + GEMM + dequant/bias)."""
    _check_ext_loaded()
    return int4_int8_ext.linear_int4_int8(x_fp32, w_packed, float(a_scale), float(w_scale), int(qn), int(qp),
                                          bias, bool(out_dtype == torch.float16))


def conv1x1_int4_int8(x_fp32, w_packed, a_scale, w_scale, qn, qp, stride_h, stride_w, bias=None,
                      out_dtype=torch.float16):
    """Fused strided 1x1 convolution, NCHW out."""
    _check_ext_loaded()
    return int4_int8_ext.conv1x1_int4_int8(x_fp32, w_packed, float(a_scale), float(w_scale), int(qn), int(qp),
                                           int(stride_h), int(stride_w), bias,
                                           bool(out_dtype == torch.float16))
