"""LSQ-quantised ResNet-18 / ResNet-50 (torchvision structure) built from
stand-in LSQ layers.

The reference converts models of the external LSQ repository
(``lsq.models``, not vendored); its adapter only relies on the duck-typed
interface used at quant_pipeline/integration/lsq_adapter.py:83-86: a layer
with a float ``conv`` (nn.Conv2d) or ``linear`` (nn.Linear) child and
``w_quant`` / ``a_quant`` quantisers carrying the LSQ step ``s`` and the
integer range ``qn``, ``qp``. ``QuantConv2d`` / ``QuantLinear`` below
implement that interface and the LSQ fake-quant forward

    x_hat = clamp(round(x / s_a), qn_a, qp_a) * s_a
    w_hat = clamp(round(w / s_w), qn_w, qp_w) * s_w,   y = op(x_hat, w_hat)

so ``convert_lsq_modules`` converts them unchanged and their float forward
is the "LSQ native" model.

Synthetic model (the LSQ checkpoint and ImageNet are not available):
He-normal weights (fan_out, ReLU gain), LSQ step s_w = 2*mean|w|/sqrt(Qp),
activation step 0.05, BatchNorm with gamma=1, beta=0, mean=0, var=1 (to be
folded), first conv and fc with 8-bit weights, every other conv INT4.
Activation ranges: the stem sees signed images [-128, 127]; every other
layer sees post-ReLU values, coded in [0, 127].
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class LsqQuantizer(nn.Module):
    """LSQ quantiser state: learnable step ``s`` and integer range [qn, qp]."""

    def __init__(self, s: float, qn: int, qp: int):
        super().__init__()
        self.s = nn.Parameter(torch.tensor(float(s), dtype=torch.float32))
        self.qn = int(qn)
        self.qp = int(qp)

    def fake_quant(self, v: torch.Tensor) -> torch.Tensor:
        s = self.s.detach()
        return torch.clamp(torch.round(v / s), self.qn, self.qp) * s


def lsq_init_step(w: torch.Tensor, qp: int) -> float:
    """LSQ step initialisation 2 * mean|w| / sqrt(Qp)."""
    return float(2.0 * w.detach().abs().mean() / math.sqrt(qp))


class QuantConv2d(nn.Module):
    def __init__(self, cin: int, cout: int, k: int, stride: int = 1, padding: int = 0, w_bits: int = 4,
                 a_range=(0, 127), a_step: float = 0.05, bias: bool = False, groups: int = 1):
        super().__init__()
        self.conv = nn.Conv2d(cin, cout, k, stride=stride, padding=padding, bias=bias, groups=groups)
        qp_w = 2 ** (w_bits - 1) - 1
        self.w_quant = LsqQuantizer(1.0, -qp_w - 1, qp_w)
        self.a_quant = LsqQuantizer(a_step, a_range[0], a_range[1])

    def reset_step(self) -> None:
        with torch.no_grad():
            self.w_quant.s.fill_(lsq_init_step(self.conv.weight, self.w_quant.qp))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        c = self.conv
        return F.conv2d(self.a_quant.fake_quant(x), self.w_quant.fake_quant(c.weight), c.bias, c.stride,
                        c.padding, c.dilation, c.groups)


class QuantLinear(nn.Module):
    def __init__(self, fin: int, fout: int, w_bits: int = 8, a_range=(0, 127), a_step: float = 0.05,
                 bias: bool = True):
        super().__init__()
        self.linear = nn.Linear(fin, fout, bias=bias)
        qp_w = 2 ** (w_bits - 1) - 1
        self.w_quant = LsqQuantizer(1.0, -qp_w - 1, qp_w)
        self.a_quant = LsqQuantizer(a_step, a_range[0], a_range[1])

    def reset_step(self) -> None:
        with torch.no_grad():
            self.w_quant.s.fill_(lsq_init_step(self.linear.weight, self.w_quant.qp))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(self.a_quant.fake_quant(x), self.w_quant.fake_quant(self.linear.weight), self.linear.bias)


class BasicBlock(nn.Module):
    expansion = 1

    def __init__(self, cin: int, planes: int, stride: int, a_step: float):
        super().__init__()
        self.conv1 = QuantConv2d(cin, planes, 3, stride, 1, a_step=a_step)
        self.bn1 = nn.BatchNorm2d(planes)
        self.conv2 = QuantConv2d(planes, planes, 3, 1, 1, a_step=a_step)
        self.bn2 = nn.BatchNorm2d(planes)
        self.downsample = None
        if stride != 1 or cin != planes:
            self.downsample = nn.Sequential(QuantConv2d(cin, planes, 1, stride, 0, a_step=a_step),
                                            nn.BatchNorm2d(planes))

    def forward(self, x):
        out = F.relu(self.bn1(self.conv1(x)))
        out = self.bn2(self.conv2(out))
        identity = x if self.downsample is None else self.downsample(x)
        return F.relu(out + identity)


class Bottleneck(nn.Module):
    expansion = 4

    def __init__(self, cin: int, planes: int, stride: int, a_step: float):
        super().__init__()
        width = planes
        self.conv1 = QuantConv2d(cin, width, 1, 1, 0, a_step=a_step)
        self.bn1 = nn.BatchNorm2d(width)
        self.conv2 = QuantConv2d(width, width, 3, stride, 1, a_step=a_step)
        self.bn2 = nn.BatchNorm2d(width)
        self.conv3 = QuantConv2d(width, planes * 4, 1, 1, 0, a_step=a_step)
        self.bn3 = nn.BatchNorm2d(planes * 4)
        self.downsample = None
        if stride != 1 or cin != planes * 4:
            self.downsample = nn.Sequential(QuantConv2d(cin, planes * 4, 1, stride, 0, a_step=a_step),
                                            nn.BatchNorm2d(planes * 4))

    def forward(self, x):
        out = F.relu(self.bn1(self.conv1(x)))
        out = F.relu(self.bn2(self.conv2(out)))
        out = self.bn3(self.conv3(out))
        identity = x if self.downsample is None else self.downsample(x)
        return F.relu(out + identity)


class LsqResNet(nn.Module):
    """torchvision-structured ResNet with LSQ layers (stem and fc 8-bit)."""

    def __init__(self, block, layers: List[int], num_classes: int = 1000, a_step: float = 0.05):
        super().__init__()
        self.conv1 = QuantConv2d(3, 64, 7, 2, 3, w_bits=8, a_range=(-128, 127), a_step=a_step)
        self.bn1 = nn.BatchNorm2d(64)
        cin = 64
        stages = []
        for i, (planes, n) in enumerate(zip((64, 128, 256, 512), layers)):
            blocks = []
            for j in range(n):
                stride = 2 if (i > 0 and j == 0) else 1
                blocks.append(block(cin, planes, stride, a_step))
                cin = planes * block.expansion
            stages.append(nn.Sequential(*blocks))
        self.layer1, self.layer2, self.layer3, self.layer4 = stages
        self.fc = QuantLinear(cin, num_classes, w_bits=8, a_range=(0, 127), a_step=a_step)

    def forward(self, x):
        x = F.relu(self.bn1(self.conv1(x)))
        x = F.max_pool2d(x, 3, 2, 1)
        x = self.layer4(self.layer3(self.layer2(self.layer1(x))))
        x = torch.flatten(F.adaptive_avg_pool2d(x, 1), 1)
        return self.fc(x)


def build_lsq_resnet(arch: str = "resnet18", num_classes: int = 1000, seed: int = 0,
                     a_step: float = 0.05) -> LsqResNet:
    """Seeded synthetic LSQ ResNet (see module docstring), eval mode, CPU."""
    if arch == "resnet18":
        model = LsqResNet(BasicBlock, [2, 2, 2, 2], num_classes, a_step)
    elif arch == "resnet50":
        model = LsqResNet(Bottleneck, [3, 4, 6, 3], num_classes, a_step)
    else:
        raise ValueError(f"unknown arch {arch}")
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, nn.Conv2d):
                fan_out = m.out_channels * m.kernel_size[0] * m.kernel_size[1]
                m.weight.normal_(0.0, math.sqrt(2.0 / fan_out), generator=gen)
            elif isinstance(m, nn.Linear):
                m.weight.normal_(0.0, math.sqrt(2.0 / m.out_features), generator=gen)
                m.bias.normal_(0.0, 0.01, generator=gen)
            elif isinstance(m, nn.BatchNorm2d):
                m.weight.fill_(1.0)
                m.bias.zero_()
                m.running_mean.zero_()
                m.running_var.fill_(1.0)
        for m in model.modules():
            if isinstance(m, (QuantConv2d, QuantLinear)):
                m.reset_step()
    return model.eval()


def synthetic_images(batch: int, seed: int = 0, size: int = 224) -> torch.Tensor:
    """N(0, 1) images [batch, 3, size, size], seeded, CPU float32."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randn((batch, 3, size, size), generator=gen, dtype=torch.float32)
