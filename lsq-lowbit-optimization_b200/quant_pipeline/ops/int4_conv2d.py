"""W4A8 conv module, API- and state_dict-compatible with
quant_pipeline/ops/int4_conv2d.py:12-201 of the reference.

State: ``weight_packed`` [O, padded_in_features/2] uint8 in the reference's
OIHW flatten order (odd C*kh*kw padded by one zero nibble, :85-109),
``w_scale`` / ``a_scale`` float32 buffers, optional float32 ``bias``.

Dispatch mirrors the reference (:145-169): 3x3/s1/p1 -> the fused 3x3 op
semantics, 1x1/s1/p0 -> the fused 1x1 op, everything else -> the
quantise/unfold/GEMM path (:171-201). All three run on the implicit-GEMM
tcgen05 kernel here (the reference's F.unfold fallback is replaced); only
geometries that kernel does not cover (dilation != 1, unequal or > 2
strides) use an explicit unfold feeding the tcgen05 GEMM. The kernel's
weight order (ky, kx, c) is derived from ``weight_packed`` on first use
and re-derived whenever the buffer changes; it is not part of the
state_dict.
"""
import math
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

import int4_int8_ext as ext
from quant_pipeline.ops.int4_int8_gemm import _check_ext_loaded
from quant_pipeline.ops.int4_linear import _scale_host
from quant_pipeline.quantization.int4_pack import pack_int4_weights


class Int4WeightInt8ActConv2d(nn.Module):
    """Conv2d with INT4 packed weights and INT8 activations."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: Tuple[int, int], stride: Tuple[int, int],
                 padding: Tuple[int, int], dilation: Tuple[int, int], groups: int, w_scale, a_scale: float,
                 a_qn: int, a_qp: int, out_dtype: torch.dtype = torch.float16, bias: bool = False) -> None:
        super().__init__()
        if groups != 1:
            raise ValueError("Only groups=1 is supported")
        self.in_channels = int(in_channels)
        self.out_channels = int(out_channels)
        self.kernel_size = tuple(int(v) for v in kernel_size)
        self.stride = tuple(int(v) for v in stride)
        self.padding = tuple(int(v) for v in padding)
        self.dilation = tuple(int(v) for v in dilation)
        self.groups = int(groups)
        self.out_dtype = out_dtype
        self.a_qn = int(a_qn)
        self.a_qp = int(a_qp)
        self.a_scale_host = float(a_scale)
        self.w_scale_host = _scale_host(w_scale)
        if self.a_qn < -128 or self.a_qp > 127:
            raise ValueError(
                f"Activation quantization range [{self.a_qn}, {self.a_qp}] does not fit int8 compute")
        self.flat_in_features = self.in_channels * self.kernel_size[0] * self.kernel_size[1]
        self.padded_in_features = self.flat_in_features + (self.flat_in_features % 2)
        self.is_pointwise = (self.kernel_size == (1, 1) and self.stride == (1, 1) and self.padding == (0, 0)
                             and self.dilation == (1, 1))
        self.is_spatial_3x3 = (self.kernel_size == (3, 3) and self.stride == (1, 1) and self.padding == (1, 1)
                               and self.dilation == (1, 1))
        ws = self.w_scale_host
        self.register_buffer("w_scale", ws.clone() if isinstance(ws, torch.Tensor)
                             else torch.tensor(ws, dtype=torch.float32))
        self.register_buffer("a_scale", torch.tensor(self.a_scale_host, dtype=torch.float32))
        self.register_buffer("weight_packed",
                             torch.zeros((self.out_channels, self.padded_in_features // 2), dtype=torch.uint8))
        if bias:
            self.bias = nn.Parameter(torch.zeros(self.out_channels, dtype=torch.float32))
        else:
            self.register_parameter("bias", None)
        self._kernel_weight = None  # (key, tensor, kind) in the conv kernel's order
        self._alpha_cache = None

    @torch.no_grad()
    def load_int4_weight(self, w_int4: torch.Tensor) -> None:
        expected = (self.out_channels, self.in_channels, self.kernel_size[0], self.kernel_size[1])
        if tuple(w_int4.shape) != expected:
            raise ValueError(f"Expected weight shape {expected}, got {tuple(w_int4.shape)}")
        if w_int4.dtype != torch.int8:
            raise TypeError("w_int4 must be int8 with values in [-8, 7]")
        w_flat = w_int4.reshape(self.out_channels, -1)
        if self.padded_in_features != self.flat_in_features:
            padded = torch.zeros((self.out_channels, self.padded_in_features), dtype=torch.int8,
                                 device=w_flat.device)
            padded[:, : self.flat_in_features] = w_flat
            w_flat = padded
        self.weight_packed.copy_(pack_int4_weights(w_flat).to(self.weight_packed.device))

    def _output_hw(self, h: int, w: int) -> Tuple[int, int]:
        h_out = math.floor((h + 2 * self.padding[0] - self.dilation[0] * (self.kernel_size[0] - 1) - 1)
                           / self.stride[0] + 1)
        w_out = math.floor((w + 2 * self.padding[1] - self.dilation[1] * (self.kernel_size[1] - 1) - 1)
                           / self.stride[1] + 1)
        return h_out, w_out

    def _kernel_supported(self) -> bool:
        kh, kw = self.kernel_size
        return (self.dilation == (1, 1) and self.stride[0] == self.stride[1] and self.stride[0] in (1, 2)
                and self.padding[0] == self.padding[1]
                and kh * kw * min(ext.conv_channels_padded(self.in_channels, self.stride[0]), 128) <= 2048)

    def _conv_weight(self):
        """(weights in the conv kernel's order, weight kind). Weights too large
        to stay resident in the kernel's shared memory are kept as int8 codes
        (ext.CONV_STREAMED_W4_BYTES), expanded once per weight version."""
        wp = self.weight_packed
        key = (wp.data_ptr(), wp._version, wp.device)
        if self._kernel_weight is None or self._kernel_weight[0] != key:
            kh, kw = self.kernel_size
            cp = ext.conv_channels_padded(self.in_channels, self.stride[0])
            w, kind = ext.repack_oihw_int4(wp.contiguous(), self.in_channels, kh, kw, cp), ext.W_INT4
            if self.out_channels * kh * kw * cp > ext.CONV_STREAMED_W4_BYTES:
                w, kind = ext.expand_int4_rows(w), ext.W_INT8
            self._kernel_weight = (key, w, kind)
        return self._kernel_weight[1], self._kernel_weight[2]

    def _alpha(self, device):
        """Scalar alpha (float) or per-channel alpha tensor. The reference's
        fused 3x3 / 1x1 ops form float(double(s_a) * double(s_w)) from the
        host floats (csrc/int4_int8_kernels.cu:345, 472); its general path
        multiplies the float32 buffers (int4_conv2d.py:192). Both are kept."""
        if not isinstance(self.w_scale_host, torch.Tensor):
            if self.is_spatial_3x3 or self.is_pointwise:
                return ext._combined_scale(self.a_scale_host, self.w_scale_host), None
            return float(self.a_scale.to(torch.float32).cpu() * self.w_scale.to(torch.float32).cpu()), None
        key = (device, self.a_scale_host)
        if self._alpha_cache is None or self._alpha_cache[0] != key:
            a = (self.a_scale_host * self.w_scale_host.to(torch.float64)).to(torch.float32).to(device)
            self._alpha_cache = (key, a)
        return 1.0, self._alpha_cache[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 4:
            raise ValueError("Input must be rank-4 [batch, channels, height, width]")
        if x.shape[1] != self.in_channels:
            raise ValueError(f"Input channels mismatch: expected {self.in_channels}, got {x.shape[1]}")
        _check_ext_loaded()
        x = x.contiguous().to(torch.float32)
        alpha_s, alpha_t = self._alpha(x.device)
        if self._kernel_supported():
            kh, kw = self.kernel_size
            # Padding of the fused 3x3 op quantises 0.0 (csrc/int4_int8_kernels.cu:242-250);
            # the unfold path pads the codes with 0 (int4_conv2d.py:172-181).
            w, kind = self._conv_weight()
            return ext.conv_nchw(x, w, kind, self.in_channels, kh, kw, self.stride[0],
                                 self.padding[0], self.a_scale_host, self.a_qn, self.a_qp, alpha_scalar=alpha_s,
                                 alpha=alpha_t, bias=self.bias, out_dtype=self.out_dtype,
                                 pad_code_of_zero=self.is_spatial_3x3)
        return self._forward_unfold(x, alpha_s, alpha_t)

    def _forward_unfold(self, x: torch.Tensor, alpha_s: float, alpha_t) -> torch.Tensor:
        """Explicit lowering for geometries outside the implicit-GEMM kernel,
        same arithmetic as the reference's general path."""
        n, _, h, w = x.shape
        h_out, w_out = self._output_hw(h, w)
        xq = ext.quantize_nchw_to_nhwc(x, self.a_scale_host, self.a_qn, self.a_qp, self.in_channels)
        xq = xq.permute(0, 3, 1, 2).to(torch.float32)  # exact small integers
        cols = F.unfold(xq, kernel_size=self.kernel_size, dilation=self.dilation, padding=self.padding,
                        stride=self.stride).transpose(1, 2).reshape(-1, self.flat_in_features)
        kp = max(32, ext._round_up(self.padded_in_features, 32))
        a = torch.zeros((cols.shape[0], kp), dtype=torch.int8, device=x.device)
        a[:, : self.flat_in_features] = cols.to(torch.int8)
        wp = ext._padded_operand(self.weight_packed.contiguous(), kp // 2)
        y = torch.empty((cols.shape[0], self.out_channels), dtype=torch.float32, device=x.device)
        epi = ext.make_epilogue(ext.OUT_F32, alpha=alpha_t, alpha_scalar=alpha_s, beta=self.bias)
        ext.gemm(a, wp, ext.W_INT4, kp, epi, y)
        y = y.view(n, h_out * w_out, self.out_channels).transpose(1, 2).reshape(n, self.out_channels, h_out, w_out)
        return y.to(self.out_dtype)
