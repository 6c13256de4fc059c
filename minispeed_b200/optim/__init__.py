from .adam import FlatAdam
from .scheduler import ConstantLR, WarmupDecayLR, WarmupLR, build_scheduler

__all__ = ["FlatAdam", "WarmupLR", "WarmupDecayLR", "ConstantLR", "build_scheduler"]
