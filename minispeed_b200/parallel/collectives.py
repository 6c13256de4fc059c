"""Gradient-reduction and parameter-gather strategies of the step pipeline.

The optimizer asks a strategy for three things per parameter group:

* ``reduce_grads``: turn this rank's model-dtype gradient arena into the
  gradient its AdamW shard needs, returning ``(tensor, mul)`` where the true
  averaged, unscaled gradient is ``tensor * mul``;
* ``stats_need_allreduce``: whether the per-rank statistics cover only a
  shard (then the flag and sum of squares are summed over ranks);
* ``gather_params``/``gather_shards``: bring the updated model-dtype shards
  of every rank into every rank's parameter arena.

Strategies:

* :class:`LocalCollectives` - world size 1: the gradient arena is used in
  place (unscale folded into the kernels' ``mul``), no communication.
* :class:`LibraryCollectives` - ``torch.distributed`` (NCCL on GPUs, gloo on
  CPU or when ranks share a GPU).  fp32 reduction like the reference
  (``zero/stage_1_and_2.py:87-102``), model-dtype parameter all-gather.
* :class:`minispeed_b200.parallel.fused.FusedCollectives` - in-kernel NVLink
  peer loads/stores (one rank per GPU of one node).

Reference: the collectives of ``minispeed/comm.py:94-141`` (``barrier``,
``all_reduce``, ``all_reduce_flag``, ``reduce_scatter``, ``all_gather_flat``,
``broadcast``) as used by ``zero/stage_1_and_2.py:80-131`` (sync, reduce,
clip, step) and ``zero/stage_3.py:68-100`` (gather / free parameters).
"""

from __future__ import annotations

from typing import Tuple

import torch
import torch.distributed as dist

from .. import comm
from ..flat import FlatParamGroup
from ..ops import kernels


class LocalCollectives:
    name = "local"

    def __init__(self, world_size: int = 1, rank: int = 0):
        self.world_size = 1
        self.rank = 0

    def attach(self, groups, zero_stage: int) -> None:
        pass

    def reduce_grads(self, g: FlatParamGroup, arena: torch.Tensor, inv_scale: float,
                     stats=None) -> Tuple[torch.Tensor, float, bool]:
        return arena[g.shard_start:g.shard_end], inv_scale, False

    def stats_need_allreduce(self, stage: int) -> bool:
        return False

    def all_reduce_stats(self, out: torch.Tensor) -> None:
        pass

    def fanout(self, g: FlatParamGroup):
        return None

    def gather_params(self, g: FlatParamGroup) -> None:
        pass

    def end_step(self) -> None:
        pass

    def check(self) -> None:
        pass

    def gather_shards(self, g: FlatParamGroup) -> None:
        """Stage 3: ``param_arena`` <- all ranks' ``param_shard``."""
        g.param_arena.copy_(g.param_shard)

    def gather_masters(self, g: FlatParamGroup) -> None:
        pass

    def close(self) -> None:
        pass


class LibraryCollectives:
    """NCCL/gloo collectives through ``torch.distributed``."""

    def __init__(self, world_size: int, rank: int):
        self.world_size = world_size
        self.rank = rank
        self.name = dist.get_backend()
        self._rs_out = {}

    def _shard_out(self, g: FlatParamGroup) -> torch.Tensor:
        if g.zero_stage >= 2:
            return g.grad_shard
        key = id(g)
        buf = self._rs_out.get(key)
        if buf is None or buf.numel() != g.shard_size:
            buf = torch.zeros(g.shard_size, dtype=torch.float32, device=g.device)
            self._rs_out[key] = buf
        return buf

    def attach(self, groups, zero_stage: int) -> None:
        pass

    def fanout(self, g: FlatParamGroup):
        return None

    def end_step(self) -> None:
        pass

    def check(self) -> None:
        pass

    def reduce_grads(self, g: FlatParamGroup, arena: torch.Tensor, inv_scale: float,
                     stats=None) -> Tuple[torch.Tensor, float, bool]:
        full = g._grad
        if full is None:
            full = torch.empty(g.numel_padded, dtype=torch.float32, device=g.device)
        kernels.cast_scale(arena, full, inv_scale)   # unscale before the reduction
        if g.zero_stage == 0:
            dist.all_reduce(full)
            g._grad = full
            return full, 1.0 / self.world_size, False
        out = self._shard_out(g)
        comm.reduce_scatter(out, full)
        g._grad = None if g.zero_stage >= 3 else full
        return out, 1.0 / self.world_size, False

    def stats_need_allreduce(self, stage: int) -> bool:
        return stage >= 1

    def all_reduce_stats(self, out: torch.Tensor) -> None:
        dist.all_reduce(out[:2])

    def _gather_into(self, full: torch.Tensor, shard: torch.Tensor) -> None:
        # ``shard`` is this rank's slice of ``full``: NCCL gathers in place,
        # gloo needs a separate input
        comm.all_gather_flat(full, shard if (full.is_cuda and self.name == "nccl")
                             else shard.clone())

    def gather_params(self, g: FlatParamGroup) -> None:
        arena = g.param_arena
        self._gather_into(arena, arena[g.shard_start:g.shard_end])

    def gather_shards(self, g: FlatParamGroup) -> None:
        comm.all_gather_flat(g.param_arena, g.param_shard)

    def gather_masters(self, g: FlatParamGroup) -> None:
        if g._partitioned:
            return
        self._gather_into(g.data, g.data[g.shard_start:g.shard_end])

    def close(self) -> None:
        self._rs_out.clear()
