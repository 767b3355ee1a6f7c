"""W4A8 inference pipeline, API-compatible with the reference's
``quant_pipeline`` package (ops, quantization, integration) and backed by
the sm_100a kernels of ``libw4a8.so``."""
