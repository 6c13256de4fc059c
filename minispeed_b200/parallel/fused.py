"""Fused in-kernel NVLink collectives of the optimizer step.

One rank per GPU of one node.  At attach time every flat group's
model-dtype gradient arena and parameter arena (stage 3: parameter shard)
are re-homed into this rank's :class:`~.peer.PeerHeap`, so the arenas that
autograd accumulates into and that the model reads are directly addressable
by every peer.  A step then runs, per rank, on one stream:

1. ``peer_barrier``: every rank finished its backward (its gradient arena is
   final);
2. ``rs_stats`` per group: the rank's shard of the sum of every peer's
   gradient arena, scaled by 1/(loss_scale*W), in fp32, fused with the
   per-block sum of squares and inf/nan flag (stage 0: the reduced slice is
   also stored into every peer's full fp32 gradient: a two-shot all-reduce);
3. ``stats_exchange``: the global flag and sum of squares, identical on all
   ranks (summed in rank order); it also proves every peer finished reading
   this rank's gradient arena;
4. ``adamw_fanout`` per group (stages 1-2): AdamW on the shard, storing the
   cast parameters into every rank's parameter arena (stage 0/3: local);
5. ``peer_barrier``: every parameter store has landed before any rank's
   next forward.

Bytes over NVLink per rank and step: (W-1)/W * N * 2 for the gradient
(16-bit operands, fp32 accumulation in registers) and (W-1)/W * N * 2 for
the parameters, against (W-1)/W * N * 4 each for the reference's fp32 NCCL
reduce-scatter and all-gather.

Every wait in these kernels is bounded (``b200.wait_timeout_ms``); a
timeout is recorded in a status word that :meth:`check` turns into
:class:`CommTimeoutError` on the host.
"""

from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch

from .. import comm
from ..flat import FlatParamGroup
from ..ops import _ext
from .peer import DTYPE_CODE, PeerHeap


class CommTimeoutError(RuntimeError):
    """A peer did not arrive at a device-side barrier within the limit."""


def supported(device: torch.device) -> Tuple[bool, str]:
    if device.type != "cuda":
        return False, "fused collectives need CUDA devices"
    if not comm.is_distributed():
        return False, "no process group"
    world = comm.get_world_size()
    local = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    if local != world:
        return False, "ranks span more than one node"
    if torch.distributed.get_backend() != "nccl":
        return False, "ranks share a GPU (gloo backend)"
    if not _ext.available():
        return False, "minispeed_b200._C not built"
    n = torch.cuda.device_count()
    if n < world:
        return False, "fewer visible GPUs than ranks"
    for q in range(n):
        if q != device.index and not torch.cuda.can_device_access_peer(device.index, q):
            return False, f"no peer access from GPU {device.index} to GPU {q}"
    return True, ""


class FusedCollectives:
    name = "fused-nvlink"

    def __init__(self, world_size: int, rank: int, device: torch.device, options=None):
        self.world_size = world_size
        self.rank = rank
        self.device = torch.device(device)
        self.timeout_s = (options.wait_timeout_ms / 1000.0) if options is not None else 10.0
        self.heap: Optional[PeerHeap] = None
        self.groups: List[FlatParamGroup] = []
        self.stage = 0
        self.epoch = 0
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._shard32 = {}
        self._step_open = False

    # ------------------------------------------------------------ set-up
    def attach(self, groups: List[FlatParamGroup], zero_stage: int) -> None:
        """Move every group's arenas into the peer heap (collective)."""
        self.groups = groups
        self.stage = zero_stage
        regions = []
        for i, g in enumerate(groups):
            esz = torch.empty((), dtype=g.param_dtype).element_size()
            regions.append((f"grad{i}", g.numel_padded * esz))
            if g._partitioned:
                regions.append((f"pshard{i}", g.shard_size * esz))
            else:
                regions.append((f"param{i}", g.numel_padded * esz))
            if zero_stage == 0:
                regions.append((f"grad32_{i}", g.numel_padded * 4))
        self.heap = PeerHeap(self.device, regions, self.rank, self.world_size)
        for i, g in enumerate(groups):
            with torch.no_grad():
                if g._partitioned:
                    shard = self.heap.view(f"pshard{i}", g.param_dtype, g.shard_size)
                    shard.copy_(g.param_shard)
                    g.param_shard = shard
                    if g.param_arena is None:
                        g._bind_placeholders()
                else:
                    arena = self.heap.view(f"param{i}", g.param_dtype, g.numel_padded)
                    arena.copy_(g.param_arena)
                    g._bind_full(arena)
                ga = self.heap.view(f"grad{i}", g.param_dtype, g.numel_padded)
                ga.zero_()
                g.grad_arena = ga
                g._arena_pinned = True
                if g.param_arena is not None:
                    g.bind_grads()
                if zero_stage == 0:
                    g._grad = self.heap.view(f"grad32_{i}", torch.float32, g.numel_padded)
        torch.cuda.synchronize(self.device)
        self.barrier()

    def _next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def barrier(self) -> None:
        _ext.get().peer_barrier(self.heap.heaps, self.heap.sync_off, self.rank,
                                self.world_size, self._next_epoch(), self.timeout_s, self.status)

    # ------------------------------------------------------------- step
    def _shard_out(self, i: int, g: FlatParamGroup) -> torch.Tensor:
        if self.stage >= 2:
            return g.grad_shard
        buf = self._shard32.get(i)
        if buf is None:
            buf = self._shard32[i] = torch.zeros(g.shard_size, dtype=torch.float32,
                                                 device=self.device)
        return buf

    def reduce_grads(self, g: FlatParamGroup, arena: torch.Tensor, inv_scale: float, stats=None):
        i = self.groups.index(g)
        if not self._step_open:
            self.barrier()          # every rank's gradient arena is final
            self._step_open = True
        if g.grad_arena is not arena:
            raise RuntimeError("gradient arena left the peer heap")
        if self.stage == 0:
            # two-shot all-reduce: reduce slice `rank`, store it to every peer
            s0 = self.rank * g.shard_size
            out = g._grad[s0:s0 + g.shard_size]
        else:
            s0 = g.shard_start
            out = self._shard_out(i, g)
        esz = arena.element_size()
        aligned = (s0 * esz) % 16 == 0 and (self.heap.offsets[f"grad{i}"] % 16) == 0
        fan = self.heap.offsets[f"grad32_{i}"] if self.stage == 0 else -1
        left = stats.partials.numel() - stats.used
        nb = _ext.get().rs_stats(self.heap.heaps, self.heap.offsets[f"grad{i}"],
                                 DTYPE_CODE[arena.dtype], s0, out, self.world_size,
                                 inv_scale / self.world_size, fan, stats.partials, stats.flags,
                                 stats.used, min(left, 148 * 8), aligned)
        stats.used += int(nb)
        if self.stage == 0:
            return g._grad, 1.0, True
        return out, 1.0, True

    def stats_need_allreduce(self, stage: int) -> bool:
        return True

    def all_reduce_stats(self, out: torch.Tensor, max_norm: Optional[float] = None) -> None:
        _ext.get().stats_exchange(self.heap.heaps, self.heap.sync_off, self.rank,
                                  self.world_size, self._next_epoch(), out,
                                  float(max_norm) if max_norm else 0.0, self.timeout_s,
                                  self.status)

    def fanout(self, g: FlatParamGroup):
        """Target of the fused AdamW + all-gather for stages 1-2."""
        if not (1 <= self.stage <= 2):
            return None
        i = self.groups.index(g)
        return (self.heap.heaps, self.heap.offsets[f"param{i}"], DTYPE_CODE[g.param_dtype],
                g.shard_start, self.world_size)

    def gather_params(self, g: FlatParamGroup) -> None:
        """Stages 1-2: the parameters were stored to every rank by AdamW."""

    def end_step(self) -> None:
        self.barrier()              # every parameter store has landed
        self._step_open = False

    def gather_shards(self, g: FlatParamGroup) -> None:
        i = self.groups.index(g)
        _ext.get().gather_pull(self.heap.heaps, self.heap.offsets[f"pshard{i}"], g.shard_size,
                               self.world_size, g.param_arena)

    def gather_masters(self, g: FlatParamGroup) -> None:
        if g._partitioned:
            return
        torch.distributed.all_gather_into_tensor(g.data, g.data[g.shard_start:g.shard_end])

    def check(self) -> None:
        code = int(self.status[0].item())
        if code:
            self.status.zero_()
            raise CommTimeoutError(f"peer wait expired (status 0x{code:x}); a rank stopped "
                                   "participating in the step")

    # -------------------------------------------------------------- exit
    def close(self) -> None:
        """Move the arenas back to ordinary allocations and unmap the heap."""
        if self.heap is None:
            return
        torch.cuda.synchronize(self.device)
        comm.barrier()
        with torch.no_grad():
            for g in self.groups:
                if g._partitioned:
                    g.param_shard = g.param_shard.clone()
                    if g.param_arena is None:
                        g._bind_placeholders()
                    else:
                        g._bind_full(g.param_arena.clone())
                else:
                    g._bind_full(g.param_arena.clone())
                if g.grad_arena is not None:
                    g.grad_arena = g.grad_arena.clone()
                    g._arena_pinned = False
                    if g.param_arena is not None:
                        g.bind_grads()
                if self.stage == 0 and g._grad is not None:
                    g._grad = g._grad.clone()
        comm.barrier()
        self.heap.close()
        self.heap = None
