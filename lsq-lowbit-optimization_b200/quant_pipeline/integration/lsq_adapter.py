"""LSQ checkpoint conversion, API-compatible with
quant_pipeline/integration/lsq_adapter.py:1-245 of the reference.

An LSQ quantised layer is duck-typed as a module with ``w_quant`` and
``a_quant`` quantisers (attributes ``s``, ``qn``, ``qp``) and a child
``linear`` (nn.Linear) or ``conv`` (nn.Conv2d). Conversion quantises the
float weight with the LSQ rule clamp(round(w / s_w), -8, 7) and swaps in
the Int4 module carrying the packed weight, the step sizes and the bias.
Layers whose weight range is not signed INT4 (the 8-bit first conv / fc
of LSQ) are skipped, exactly like the reference. A quantiser whose step
``s`` holds one value per output channel produces a per-channel weight
scale (an extension; scalar steps behave exactly as in the reference).
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import List, Optional

import torch
import torch.nn as nn

from quant_pipeline.ops import Int4WeightInt8ActConv2d, Int4WeightInt8ActLinear


@dataclass
class ConversionResult:
    name: str
    module_type: str
    converted: bool
    reason: str


def _resolve_num_classes(state: dict, default: int = 1000) -> int:
    for key in ("fc.weight", "fc.linear.weight"):
        if key in state:
            return int(state[key].shape[0])
    return default


def _is_lsq_checkpoint(state: dict) -> bool:
    return any(".w_quant." in k or ".a_quant." in k or k.endswith(".conv.weight") for k in state)


def build_lsq_model_from_ckpt(lsq_root, ckpt_path, w_bits: int = 4, a_bits: int = 4, first_last_bits: int = 8,
                              disable_first_last_8bit: bool = False, signed_input_first_layer: bool = False,
                              num_classes: Optional[int] = None) -> nn.Module:
    """Builds the LSQ pre-activation ResNet-18 from the external LSQ
    repository at ``lsq_root`` and loads ``ckpt_path`` (``ckpt["model"]`` or
    a raw state_dict), as lsq_adapter.py:36-80 does."""
    import sys

    lsq_root = Path(lsq_root).resolve()
    if not lsq_root.exists():
        raise FileNotFoundError(f"LSQ root not found: {lsq_root}")
    if str(lsq_root) not in sys.path:
        sys.path.insert(0, str(lsq_root))
    from lsq.models import LSQConfig, apply_lsq_quantization, preact_resnet18  # external dependency

    ckpt = torch.load(str(ckpt_path), map_location="cpu")
    state = ckpt["model"] if isinstance(ckpt, dict) and "model" in ckpt else ckpt
    if num_classes is None:
        num_classes = _resolve_num_classes(state)
    model = preact_resnet18(num_classes=num_classes)
    if _is_lsq_checkpoint(state):
        apply_lsq_quantization(model, LSQConfig(w_bits=w_bits, a_bits=a_bits, first_last_bits=first_last_bits,
                                                quantize_first_last_8bit=not disable_first_last_8bit,
                                                signed_input_first_layer=signed_input_first_layer))
    model.load_state_dict(state, strict=True)
    return model


def _is_lsq_quant_module(module: nn.Module) -> bool:
    return hasattr(module, "w_quant") and hasattr(module, "a_quant") and (
        hasattr(module, "linear") or hasattr(module, "conv"))


def _replace_module(root: nn.Module, name: str, module: nn.Module) -> None:
    parent = root
    *path, leaf = name.split(".")
    for part in path:
        parent = getattr(parent, part)
    setattr(parent, leaf, module)


def _get_quant_range(quantizer: nn.Module) -> tuple[int, int]:
    return int(getattr(quantizer, "qn")), int(getattr(quantizer, "qp"))


def _quantize_tensor(v: torch.Tensor, scale, qn: int, qp: int) -> torch.Tensor:
    """LSQ weight codes clamp(round(v / s), qn, qp) (lsq_adapter.py:103-104);
    ``scale`` is a float or a per-output-channel tensor."""
    if isinstance(scale, torch.Tensor):
        scale = scale.to(v.device, v.dtype).reshape(-1, *([1] * (v.dim() - 1)))
    return torch.clamp(torch.round(v / scale), qn, qp).to(torch.int8)


def _step(quantizer: nn.Module):
    s = torch.clamp(quantizer.s.detach(), min=1e-8)
    return float(s.item()) if s.numel() == 1 else s.to(torch.float32).reshape(-1).cpu()


def _check_ranges(w_quant, a_quant) -> Optional[str]:
    w_qn, w_qp = _get_quant_range(w_quant)
    a_qn, a_qp = _get_quant_range(a_quant)
    if (w_qn, w_qp) != (-8, 7):
        return f"weight range [{w_qn}, {w_qp}] is not signed INT4"
    if a_qn < -128 or a_qp > 127:
        return f"activation range [{a_qn}, {a_qp}] does not fit int8 compute"
    return None


def _convert_quant_linear_module(name: str, module: nn.Module):
    if not isinstance(module.linear, nn.Linear):
        return None, "linear child is not nn.Linear"
    linear = module.linear
    reason = _check_ranges(module.w_quant, module.a_quant)
    if reason:
        return None, reason
    if linear.in_features % 2 != 0:
        return None, "in_features is odd and current int4 linear path cannot pack it"
    w_scale, a_scale = _step(module.w_quant), _step(module.a_quant)
    if isinstance(a_scale, torch.Tensor):
        return None, "per-channel activation step is not supported"
    a_qn, a_qp = _get_quant_range(module.a_quant)
    fused = Int4WeightInt8ActLinear(in_features=linear.in_features, out_features=linear.out_features,
                                    w_scale=w_scale, a_scale=a_scale, a_qn=a_qn, a_qp=a_qp,
                                    out_dtype=torch.float32, bias=linear.bias is not None).to(linear.weight.device)
    fused.load_int4_weight(_quantize_tensor(linear.weight.detach(), w_scale, -8, 7))
    if linear.bias is not None:
        fused.bias.data.copy_(linear.bias.detach().to(fused.bias.dtype))
    return fused, "converted"


def _convert_quant_conv_module(name: str, module: nn.Module):
    if not isinstance(module.conv, nn.Conv2d):
        return None, "conv child is not nn.Conv2d"
    conv = module.conv
    reason = _check_ranges(module.w_quant, module.a_quant)
    if reason:
        return None, reason
    if conv.groups != 1:
        return None, "grouped convolution is not supported"
    w_scale, a_scale = _step(module.w_quant), _step(module.a_quant)
    if isinstance(a_scale, torch.Tensor):
        return None, "per-channel activation step is not supported"
    a_qn, a_qp = _get_quant_range(module.a_quant)
    fused = Int4WeightInt8ActConv2d(in_channels=conv.in_channels, out_channels=conv.out_channels,
                                    kernel_size=conv.kernel_size, stride=conv.stride, padding=conv.padding,
                                    dilation=conv.dilation, groups=conv.groups, w_scale=w_scale, a_scale=a_scale,
                                    a_qn=a_qn, a_qp=a_qp, out_dtype=torch.float32,
                                    bias=conv.bias is not None).to(conv.weight.device)
    fused.load_int4_weight(_quantize_tensor(conv.weight.detach(), w_scale, -8, 7))
    if conv.bias is not None:
        fused.bias.data.copy_(conv.bias.detach().to(fused.bias.dtype))
    return fused, "converted"


@torch.no_grad()
def convert_lsq_modules(model: nn.Module, only_names: Optional[List[str]] = None, convert_linear: bool = True,
                        convert_conv: bool = False) -> List[ConversionResult]:
    """Replaces LSQ QuantLinear / QuantConv2d modules in place
    (lsq_adapter.py:192-234); returns one result per LSQ module seen."""
    results: List[ConversionResult] = []
    for name, module in list(model.named_modules()):
        if only_names is not None and name not in only_names:
            continue
        if not _is_lsq_quant_module(module):
            continue
        converted, reason, module_type = None, "unsupported module", type(module).__name__
        if hasattr(module, "linear"):
            module_type = "QuantLinear"
            if convert_linear:
                converted, reason = _convert_quant_linear_module(name, module)
            else:
                reason = "linear conversion disabled"
        elif hasattr(module, "conv"):
            module_type = "QuantConv2d"
            if convert_conv:
                converted, reason = _convert_quant_conv_module(name, module)
            else:
                reason = "conv conversion disabled"
        if converted is not None:
            _replace_module(model, name, converted)
        results.append(ConversionResult(name=name, module_type=module_type, converted=converted is not None,
                                        reason=reason))
    return results


@torch.no_grad()
def convert_quant_linear_modules(model: nn.Module, only_names: Optional[List[str]] = None) -> List[str]:
    """Linear-only conversion; returns the converted module names."""
    results = convert_lsq_modules(model, only_names=only_names, convert_linear=True, convert_conv=False)
    return [r.name for r in results if r.converted]
