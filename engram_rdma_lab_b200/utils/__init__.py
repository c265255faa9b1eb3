from .env import KNOBS, EnvOverride, describe_knobs
from .event import EventOverlap
from .math import align, ceil_div

__all__ = ["KNOBS", "EnvOverride", "describe_knobs", "EventOverlap", "align", "ceil_div"]
