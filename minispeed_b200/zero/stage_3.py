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

from typing import List, Optional, Tuple

import torch

from ..flat import FlatParamGroup
from .stage_1_and_2 import ZeROOptimizer


class ZeROStage3Optimizer(ZeROOptimizer):
    def __init__(self, flat_groups: List[FlatParamGroup], option_groups: List[dict],
                 collectives=None):
        super().__init__(flat_groups, option_groups, zero_stage=3, collectives=collectives)
        self._gathered = False
        # layer-wise gather (fused collectives): arena ranges per model block
        self._layer_plan: Optional[List[List[Tuple[int, int, int]]]] = None
        self._layer_rest: Optional[List[List[Tuple[int, int]]]] = None
        self._layer_events: Optional[list] = None
        self.gather_stream = None

    @property
    def params_gathered(self) -> bool:
        return self._gathered

    def plan_layer_gather(self, blocks: List[List[torch.nn.Parameter]]) -> bool:
        """Gather each block's parameters just ahead of its forward instead
        of the whole model before the first block (needs the fused NVLink
        collectives; each block's parameters must be one contiguous arena
        range per group)."""
        if not hasattr(self.coll, "gather_range") or self.stats.device.type != "cuda":
            return False
        where = {}
        for gi, g in enumerate(self.flat_groups):
            for p, off, n in zip(g.params, g._offsets_int, g._numels):
                where[id(p)] = (gi, off, n)
        plan, seen = [], set()
        covered = [[] for _ in self.flat_groups]
        for params in blocks:
            spans = {}
            for p in params:
                if id(p) not in where or id(p) in seen:
                    return False
                seen.add(id(p))
                gi, off, n = where[id(p)]
                lo, hi, tot = spans.get(gi, (off, off + n, 0))
                spans[gi] = (min(lo, off), max(hi, off + n), tot + n)
            if any(hi - lo != tot for lo, hi, tot in spans.values()):
                return False
            plan.append([(gi, lo, hi) for gi, (lo, hi, _) in sorted(spans.items())])
            for gi, (lo, hi, _) in spans.items():
                covered[gi].append((lo, hi))
        rest = []
        for gi, g in enumerate(self.flat_groups):
            r, cur = [], 0
            for lo, hi in sorted(covered[gi]):
                if lo > cur:
                    r.append((cur, lo))
                cur = max(cur, hi)
            if cur < g.numel_padded:
                r.append((cur, g.numel_padded))
            rest.append(r)
        self._layer_plan, self._layer_rest = plan, rest
        self.gather_stream = torch.cuda.Stream(self.stats.device)
        return True

    @torch.no_grad()
    def gather_parameters(self, layerwise: bool = False) -> None:
        """Collective: materialize the full params on every rank.  With
        ``layerwise`` (the engine's forward) only the parameters outside the
        model blocks are gathered here; each block's come from
        :meth:`layer_ready`, one block ahead of its forward."""
        if self._gathered:
            return
        lazy = layerwise and self._layer_plan is not None
        for gi, g in enumerate(self.flat_groups):
            g.materialize_params()
            if lazy:
                for lo, hi in self._layer_rest[gi]:
                    self.coll.gather_range(g, lo, hi)
            else:
                self.coll.gather_shards(g)
            if torch.is_grad_enabled() or g._arena_pinned:
                g.ensure_grad_arena()
        if lazy:
            self._layer_events = [None] * len(self._layer_plan)
            self.gather_stream.wait_stream(torch.cuda.current_stream(self.stats.device))
            self._launch_layer(0)
        self._gathered = True

    def _launch_layer(self, k: int) -> None:
        if k >= len(self._layer_plan) or self._layer_events[k] is not None:
            return
        with torch.cuda.stream(self.gather_stream):
            for gi, lo, hi in self._layer_plan[k]:
                self.coll.gather_range(self.flat_groups[gi], lo, hi)
            ev = torch.cuda.Event()
            ev.record()
        self._layer_events[k] = ev

    def layer_ready(self, k: int) -> None:
        """Forward pre-hook of block k: wait for its parameters, start
        gathering block k+1's."""
        if not self._gathered or self._layer_events is None:
            return
        self._launch_layer(k)
        torch.cuda.current_stream(self.stats.device).wait_event(self._layer_events[k])
        self._launch_layer(k + 1)

    def _finish_layer_gather(self) -> None:
        if self._layer_events is not None:
            for k in range(len(self._layer_plan)):
                self._launch_layer(k)
            torch.cuda.current_stream(self.stats.device).wait_stream(self.gather_stream)
            self._layer_events = None

    def boundary_step(self, loss_scale, max_norm):
        self._finish_layer_gather()
        return super().boundary_step(loss_scale, max_norm)

    @torch.no_grad()
    def free_parameters(self, refresh: bool = True) -> None:
        """Drop the full params back to their locally owned slices."""
        if not self._gathered:
            return
        self._finish_layer_gather()
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
