from .lsq_adapter import ConversionResult, build_lsq_model_from_ckpt, convert_lsq_modules, convert_quant_linear_modules

__all__ = [
    "ConversionResult",
    "build_lsq_model_from_ckpt",
    "convert_lsq_modules",
    "convert_quant_linear_modules",
]
