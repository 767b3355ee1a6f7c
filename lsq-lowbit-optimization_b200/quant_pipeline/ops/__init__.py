from .int4_conv2d import Int4WeightInt8ActConv2d
from .int4_int8_gemm import int8_int8_gemm, int4_int8_gemm
from .int4_linear import Int4WeightInt8ActLinear

__all__ = [
    "int8_int8_gemm",
    "int4_int8_gemm",
    "Int4WeightInt8ActConv2d",
    "Int4WeightInt8ActLinear",
]
