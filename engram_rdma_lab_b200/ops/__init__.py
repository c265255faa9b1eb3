from .fp8 import E4M3_MAX, calc_diff, dequantize_fp8_blockwise, quantize_fp8_blockwise
from .pack import route_pack, route_pack_reference

__all__ = ["E4M3_MAX", "calc_diff", "dequantize_fp8_blockwise", "quantize_fp8_blockwise", "route_pack",
           "route_pack_reference"]
