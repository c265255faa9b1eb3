from .env import KNOBS, EnvOverride, describe_knobs
from .event import EventOverlap
from .math import align, calc_diff, ceil_div, count_bytes, hash_tensors, safe_div

__all__ = ["KNOBS", "EnvOverride", "describe_knobs", "EventOverlap", "align", "calc_diff", "ceil_div", "count_bytes", "hash_tensors", "safe_div"]
