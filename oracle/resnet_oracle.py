"""CPU oracle of the LSQ-converted ResNet forward — TEST INFRASTRUCTURE ONLY.

Integer semantics of a converted model (the reference's Int4 modules:
quantise the fp32 input, integer conv, float epilogue;
quant_pipeline/ops/int4_conv2d.py:171-201) with inference BatchNorm folded
into the per-channel epilogue:

    m[c]     = gamma[c] / sqrt(var[c] + eps)                         (float64)
    alpha[c] = float32((s_a * s_w) * m[c])                            (float64 -> f32)
    beta[c]  = float32((bias[c] - mean[c]) * m[c] + bn_beta[c])
    y        = f32(acc) * alpha + beta  (+ identity)  (ReLU)          (float32 ops)

Weights are coded clamp(round(w / s_w), qn_w, qp_w) (lsq_adapter.py:103-104)
and activations clamp(round(x / s_a), qn_a, qp_a) at each layer's input.
Pooling: 3x3/s2/p1 max (padding never wins) and a sequential float32 mean.
Reads only the float parameters of the model object it is given.
"""
from __future__ import annotations

import math

import numpy as np

from oracle import oracle as orc


def _np(t):
    return t.detach().cpu().numpy()


def layer_params(qconv, bn=None):
    """Integer weights (OHWI int8), activation quant params and the folded
    epilogue (alpha, beta) of an LSQ conv / linear + optional BN."""
    is_conv = hasattr(qconv, "conv")
    lin = qconv.conv if is_conv else qconv.linear
    w = _np(lin.weight).astype(np.float32)
    s_w = float(qconv.w_quant.s.detach())
    s_a = float(qconv.a_quant.s.detach())
    wq = orc.quantize(w, s_w, qconv.w_quant.qn, qconv.w_quant.qp)
    o = w.shape[0]
    bias = _np(lin.bias).astype(np.float64) if lin.bias is not None else np.zeros(o)
    if bn is not None:
        mult = _np(bn.weight).astype(np.float64) / np.sqrt(_np(bn.running_var).astype(np.float64) + bn.eps)
        shift = (bias - _np(bn.running_mean).astype(np.float64)) * mult + _np(bn.bias).astype(np.float64)
    else:
        mult, shift = np.ones(o), bias
    alpha = ((np.float64(s_a) * np.float64(s_w)) * mult).astype(np.float32)
    beta = shift.astype(np.float32)
    p = dict(s_a=s_a, qn=qconv.a_quant.qn, qp=qconv.a_quant.qp, alpha=alpha, beta=beta)
    if is_conv:
        p.update(w=wq.transpose(0, 2, 3, 1), stride=lin.stride[0], pad=lin.padding[0])
    else:
        p.update(w=wq)
    return p


def conv_layer(x_nhwc: np.ndarray, p: dict, relu: bool, residual=None) -> np.ndarray:
    n, h, w, _ = x_nhwc.shape
    o, kh, kw, _ = p["w"].shape
    s, pad = p["stride"], p["pad"]
    ho = (h + 2 * pad - kh) // s + 1
    wo = (w + 2 * pad - kw) // s + 1
    xq = orc.quantize(x_nhwc, p["s_a"], p["qn"], p["qp"])
    acc = orc.conv_nhwc_s32(xq, p["w"], s, pad, pad, ho, wo)
    return orc.epilogue(acc, p["alpha"], p["beta"], residual, relu)


def block_forward(block, x: np.ndarray) -> np.ndarray:
    if block.downsample is not None:
        identity = conv_layer(x, layer_params(block.downsample[0], block.downsample[1]), relu=False)
    else:
        identity = x
    if hasattr(block, "conv3"):
        h = conv_layer(x, layer_params(block.conv1, block.bn1), relu=True)
        h = conv_layer(h, layer_params(block.conv2, block.bn2), relu=True)
        return conv_layer(h, layer_params(block.conv3, block.bn3), relu=True, residual=identity)
    h = conv_layer(x, layer_params(block.conv1, block.bn1), relu=True)
    return conv_layer(h, layer_params(block.conv2, block.bn2), relu=True, residual=identity)


def resnet_forward(model, images_nchw: np.ndarray) -> np.ndarray:
    """Logits [n, classes] float32 of the converted model on ``images``."""
    x = np.ascontiguousarray(np.asarray(images_nchw, dtype=np.float32).transpose(0, 2, 3, 1))
    x = conv_layer(x, layer_params(model.conv1, model.bn1), relu=True)
    x = orc.maxpool3x3s2(x)
    for stage in (model.layer1, model.layer2, model.layer3, model.layer4):
        for block in stage:
            x = block_forward(block, x)
    pooled = orc.avgpool(x)
    fc = layer_params(model.fc)
    q = orc.quantize(pooled, fc["s_a"], fc["qn"], fc["qp"])
    acc = orc.gemm_s32(q, fc["w"])
    return orc.epilogue(acc, fc["alpha"], fc["beta"])


def top1_agreement(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.mean(np.argmax(a, axis=1) == np.argmax(b, axis=1)))


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    """max |got - want| / max |want| (logit-scale relative error)."""
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


__all__ = ["layer_params", "conv_layer", "block_forward", "resnet_forward", "top1_agreement", "rel_err", "math"]
