from .env import EnvOverride
from .event import EventOverlap
from .math import align, calc_diff, ceil_div, count_bytes, hash_tensors, safe_div

__all__ = ["EnvOverride", "EventOverlap", "align", "calc_diff", "ceil_div", "count_bytes", "hash_tensors", "safe_div"]
