"""Signed INT4 packing, two values per byte along the last dimension.

Layout and checks follow quant_pipeline/quantization/int4_pack.py:9-50 of
the reference: element 2j is the low nibble and element 2j+1 the high
nibble of byte j, both in 4-bit two's complement. This is the on-disk
format of ``weight_packed`` buffers and the format the kernels consume.
"""
import torch


def pack_int4_weights(w_int4: torch.Tensor) -> torch.Tensor:
    """Packs int values in [-8, 7] along the last dim ([..., K] -> [..., K/2] uint8)."""
    if w_int4.dtype not in (torch.int8, torch.int16, torch.int32):
        raise TypeError(f"Expected integer tensor, got {w_int4.dtype}")
    if w_int4.shape[-1] % 2 != 0:
        raise ValueError("Last dimension K must be even for int4 packing")
    if torch.any(w_int4 < -8) or torch.any(w_int4 > 7):
        raise ValueError("INT4 tensor contains values outside [-8, 7]")
    nib = (w_int4.to(torch.int16) & 0xF).to(torch.uint8)
    return nib[..., 0::2] | (nib[..., 1::2] << 4)


def unpack_int4_weights(w_packed: torch.Tensor) -> torch.Tensor:
    """Inverse of pack_int4_weights: uint8 [..., K/2] -> int8 [..., K]."""
    if w_packed.dtype != torch.uint8:
        raise TypeError(f"Expected uint8 tensor, got {w_packed.dtype}")
    lo = ((w_packed & 0xF).to(torch.int8) << 4) >> 4
    hi = (((w_packed >> 4) & 0xF).to(torch.int8) << 4) >> 4
    return torch.stack((lo, hi), dim=-1).flatten(-2)
