"""Minimal stand-in LSQ layers for fixture generation and adapter tests.

Duck-types the interface the reference's adapter converts
(quant_pipeline/integration/lsq_adapter.py:83-86): a float ``conv`` /
``linear`` child and ``w_quant`` / ``a_quant`` quantisers with ``s``, ``qn``,
``qp``. Standalone (imports nothing from either quant_pipeline package) so
the same model can be built next to the reference and next to this
repository.
"""
import math

import torch
import torch.nn as nn


class Quantizer(nn.Module):
    def __init__(self, s, qn, qp):
        super().__init__()
        self.s = nn.Parameter(torch.tensor(float(s)))
        self.qn, self.qp = int(qn), int(qp)


class QConv(nn.Module):
    def __init__(self, cin, cout, k, stride, pad, w_range=(-8, 7), a_range=(0, 127), bias=False, groups=1):
        super().__init__()
        self.conv = nn.Conv2d(cin, cout, k, stride, pad, bias=bias, groups=groups)
        self.w_quant = Quantizer(1.0, *w_range)
        self.a_quant = Quantizer(0.05, *a_range)


class QLinear(nn.Module):
    def __init__(self, fin, fout, w_range=(-8, 7), a_range=(-127, 127), bias=True):
        super().__init__()
        self.linear = nn.Linear(fin, fout, bias=bias)
        self.w_quant = Quantizer(1.0, *w_range)
        self.a_quant = Quantizer(0.05, *a_range)


def build_standin(seed: int = 0) -> nn.Module:
    torch.manual_seed(seed)
    m = nn.Module()
    m.q1 = QConv(16, 32, 3, 1, 1, bias=True)
    m.q2 = QConv(32, 32, 3, 2, 1)
    m.q3 = QConv(3, 16, 7, 2, 3, w_range=(-128, 127), a_range=(-128, 127))
    m.q4 = QLinear(64, 10)
    m.q5 = QLinear(63, 10)
    m.q6 = QConv(16, 16, 3, 1, 1, groups=2)
    m.q7 = QConv(16, 16, 1, 1, 0, a_range=(0, 200))
    m.q8 = QConv(3, 8, 5, 1, 2, bias=True)
    with torch.no_grad():
        for mod in m.modules():
            child = getattr(mod, "conv", None) or getattr(mod, "linear", None)
            if child is not None and hasattr(mod, "w_quant"):
                qp = mod.w_quant.qp
                mod.w_quant.s.fill_(float(2 * child.weight.abs().mean() / math.sqrt(qp)))
                mod.a_quant.s.fill_(0.037 if mod.a_quant.qn < 0 else 0.05)
    return m.eval()
