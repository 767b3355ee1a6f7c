"""W4A8 linear module, API- and state_dict-compatible with
quant_pipeline/ops/int4_linear.py:8-88 of the reference.

Buffers: ``weight_packed`` [O, K/2] uint8 (int4_pack layout), ``w_scale``
and ``a_scale`` float32 (0-d, or [O] for a per-output-channel weight
scale), optional float32 ``bias`` parameter. Forward quantises the fp32
input with (a_scale, a_qn, a_qp), runs the tcgen05 W4A8 GEMM and applies
y = acc * (s_a * s_w) + bias in the GEMM epilogue.
"""
from typing import Union

import torch
import torch.nn as nn

import int4_int8_ext
from quant_pipeline.ops.int4_int8_gemm import _check_ext_loaded, linear_int4_int8
from quant_pipeline.quantization.int4_pack import pack_int4_weights


def _scale_host(scale: Union[float, torch.Tensor]):
    if isinstance(scale, torch.Tensor) and scale.numel() > 1:
        return scale.detach().to(torch.float32).cpu().reshape(-1)
    return float(scale)


class Int4WeightInt8ActLinear(nn.Module):
    """INT4 weights (packed uint8), INT8 activations, INT32 accumulation,
    FP16/FP32 dequantised output."""

    def __init__(self, in_features: int, out_features: int, w_scale, a_scale: float, a_qn: int = -127,
                 a_qp: int = 127, out_dtype: torch.dtype = torch.float16, bias: bool = False):
        super().__init__()
        if in_features % 2 != 0:
            raise ValueError("in_features must be even for INT4 packing")
        self.in_features = in_features
        self.out_features = out_features
        self.out_dtype = out_dtype
        self.a_qn = int(a_qn)
        self.a_qp = int(a_qp)
        self.a_scale_host = float(a_scale)
        self.w_scale_host = _scale_host(w_scale)
        if self.a_qn < -128 or self.a_qp > 127:
            raise ValueError(
                f"Activation quantization range [{self.a_qn}, {self.a_qp}] does not fit int8 compute")
        ws = self.w_scale_host
        self.register_buffer("w_scale", ws.clone() if isinstance(ws, torch.Tensor)
                             else torch.tensor(ws, dtype=torch.float32))
        self.register_buffer("a_scale", torch.tensor(self.a_scale_host, dtype=torch.float32))
        self.register_buffer("weight_packed", torch.zeros((out_features, in_features // 2), dtype=torch.uint8))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=torch.float32))
        else:
            self.register_parameter("bias", None)
        self._alpha_cache = None

    @torch.no_grad()
    def load_int4_weight(self, w_int4: torch.Tensor) -> None:
        if w_int4.shape != (self.out_features, self.in_features):
            raise ValueError(
                f"Expected weight shape {(self.out_features, self.in_features)}, got {tuple(w_int4.shape)}")
        if w_int4.dtype != torch.int8:
            raise TypeError("w_int4 must be int8 with values in [-8, 7]")
        self.weight_packed.copy_(pack_int4_weights(w_int4).to(self.weight_packed.device))

    def _alpha(self, device) -> torch.Tensor:
        key = (device, self.a_scale_host)
        if self._alpha_cache is None or self._alpha_cache[0] != key:
            a = (self.a_scale_host * self.w_scale_host.to(torch.float64)).to(torch.float32).to(device)
            self._alpha_cache = (key, a)
        return self._alpha_cache[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 2:
            raise ValueError("Input must be rank-2 [batch, in_features]")
        if x.shape[1] != self.in_features:
            raise ValueError(f"Input in_features mismatch: expected {self.in_features}, got {x.shape[1]}")
        x = x.contiguous().to(torch.float32)
        if not isinstance(self.w_scale_host, torch.Tensor):
            return linear_int4_int8(x, self.weight_packed.contiguous(), self.a_scale_host, self.w_scale_host,
                                    self.a_qn, self.a_qp, self.bias, self.out_dtype)
        # Per-output-channel weight scale: alpha[n] = float(s_a * s_w[n]).
        _check_ext_loaded()
        ext = int4_int8_ext
        m, k = x.shape
        out = torch.empty((m, self.out_features), dtype=self.out_dtype, device=x.device)
        if out.numel() == 0:
            return out
        kp = max(32, ext._round_up(k, 32))
        xq = ext.quantize_rows(x, self.a_scale_host, self.a_qn, self.a_qp, ldq=kp)
        wp = ext._padded_operand(self.weight_packed.contiguous(), kp // 2)
        kind = ext.OUT_F16 if self.out_dtype == torch.float16 else ext.OUT_F32
        epi = ext.make_epilogue(kind, alpha=self._alpha(x.device), beta=self.bias)
        return ext.gemm(xq, wp, ext.W_INT4, kp, epi, out)
