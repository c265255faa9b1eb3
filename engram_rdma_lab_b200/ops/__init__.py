from .fp8 import E4M3_MAX, dequantize_fp8_blockwise, quantize_fp8_blockwise

__all__ = ["E4M3_MAX", "dequantize_fp8_blockwise", "quantize_fp8_blockwise"]
