"""ZeRO stage 3: parameters are partitioned too.

Between optimizer steps each rank stores only its shard of the fp32 masters,
the matching Adam moments, its reduced gradient shard and a flat model-dtype
placeholder slice of every parameter (reference
``minispeed/zero/stage_3.py:1-126``).  The full parameters exist between
:meth:`gather_parameters` (first forward of an accumulation window, or
around checkpoint save/load) and :meth:`free_parameters` (after the step).

Differences in how it is done here:

* the gather moves model-dtype shards (2 bytes/element for fp16/bf16), not
  the fp32 masters followed by a cast: the placeholders always hold the cast
  of the masters (AdamW writes them), so the values are identical;
* after the step no placeholder refresh copy is needed, for the same reason.
"""

from __future__ import annotations

from typing import List

import torch

from ..flat import FlatParamGroup
from .stage_1_and_2 import ZeROOptimizer


class ZeROStage3Optimizer(ZeROOptimizer):
    def __init__(self, flat_groups: List[FlatParamGroup], option_groups: List[dict],
                 collectives=None):
        super().__init__(flat_groups, option_groups, zero_stage=3, collectives=collectives)
        self._gathered = False

    @property
    def params_gathered(self) -> bool:
        return self._gathered

    @torch.no_grad()
    def gather_parameters(self) -> None:
        """Collective: materialize the full params on every rank."""
        if self._gathered:
            return
        for g in self.flat_groups:
            g.materialize_params()
            self.coll.gather_shards(g)
            if torch.is_grad_enabled() or g._arena_pinned:
                g.ensure_grad_arena()
        self._gathered = True

    @torch.no_grad()
    def free_parameters(self, refresh: bool = True) -> None:
        """Drop the full params back to their locally owned slices."""
        if not self._gathered:
            return
        for g in self.flat_groups:
            g.dematerialize_params()
            if refresh:
                g.copy_flat_to_model()
        self._gathered = False

    @torch.no_grad()
    def sync_parameters(self) -> None:
        self.free_parameters()

    def sync_master_weights(self) -> None:
        """Stage 3 keeps only shards; every shard is always current."""

    @torch.no_grad()
    def step(self) -> bool:
        self.adam.step()
        return True

    @torch.no_grad()
    def reduce_gradients(self) -> None:
        super().reduce_gradients()
        for g in self.flat_groups:
            g.grad = None

    def after_step(self, applied: bool) -> None:
        # AdamW already wrote the placeholders (param_shard) when it ran;
        # on a skipped step the masters are unchanged, so neither refreshes.
        self.free_parameters(refresh=False)
