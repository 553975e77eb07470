"""Weight-only quantization: int8 quantizer and GEMV, module swap and selection rules."""
