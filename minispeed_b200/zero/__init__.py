"""ZeRO optimizers (stages 0-3) and their factory."""

from typing import List

from ..flat import FlatParamGroup
from .stage_1_and_2 import ZeROOptimizer, make_collectives
from .stage_3 import ZeROStage3Optimizer


def build_zero_optimizer(flat_groups: List[FlatParamGroup], option_groups: List[dict],
                         zero_stage: int = 0, collectives=None) -> ZeROOptimizer:
    """Stage 3 also partitions the parameters (reference ``zero/__init__.py:8-16``)."""
    if zero_stage >= 3:
        return ZeROStage3Optimizer(flat_groups, option_groups, collectives=collectives)
    return ZeROOptimizer(flat_groups, option_groups, zero_stage=zero_stage,
                         collectives=collectives)


__all__ = ["ZeROOptimizer", "ZeROStage3Optimizer", "build_zero_optimizer", "make_collectives"]
