from .engram_tables import (
    CONFIGS,
    TableSpec,
    expected_outputs,
    expected_random_init,
    make_indices,
    normal_bf16_shard,
    pattern_scales,
    pattern_shard,
    quantized_fp8_shard,
    row_pattern,
)

__all__ = [
    "CONFIGS",
    "TableSpec",
    "expected_outputs",
    "expected_random_init",
    "make_indices",
    "normal_bf16_shard",
    "pattern_scales",
    "pattern_shard",
    "quantized_fp8_shard",
    "row_pattern",
]
