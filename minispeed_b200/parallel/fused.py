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

Reference: the same step semantics as ``minispeed/engine.py:269-322``
(``_take_optimizer_step``) over ``zero/stage_1_and_2.py:87-145`` (fp32
reduce-scatter, overflow all-reduce, global norm, clip, AdamW on the shard,
all-gather), with the NCCL calls replaced by peer memory accesses.

Every wait in these kernels is bounded (``b200.wait_timeout_ms``); a
timeout is recorded in a status word that :meth:`check` turns into
:class:`CommTimeoutError` on the host.
"""

from __future__ import annotations

import os
import socket
from typing import List, Optional, Tuple

import torch

from .. import comm
from ..flat import FlatParamGroup
from ..ops import _ext
from .peer import DTYPE_CODE, PeerHeap


class CommTimeoutError(RuntimeError):
    """A peer did not arrive at a device-side barrier within the limit."""


def _device_identity(device: torch.device) -> str:
    """Host name and the GPU's UUID (its raw bytes, so that no formatting of
    the UUID object can make two GPUs look alike); the device index when the
    UUID is not available."""
    raw = getattr(getattr(torch.cuda.get_device_properties(device), "uuid", None), "bytes", None)
    try:
        key = bytes(raw).hex() if raw is not None else None
    except (TypeError, ValueError):
        key = None
    return f"{socket.gethostname()}/{key if key else 'index%d' % device.index}"


def shared_gpu(identities) -> bool:
    """True when two ranks reported the same GPU."""
    ids = list(identities)
    return len(set(ids)) != len(ids)


def supported(device: torch.device) -> Tuple[bool, str]:
    """Whether the fused NVLink collectives can serve this process group, and
    why not.  Collective when the group uses NCCL: every rank must call it."""
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
    # every rank takes part here, before any rank-dependent return: the
    # fused kernels wait on their peers, and two such waiting kernels from
    # two processes on one GPU are not guaranteed to run at the same time
    if shared_gpu(comm.all_gather_object(_device_identity(device))):
        return False, "two ranks use the same GPU"
    if not _ext.available():
        return False, "minispeed_b200._C not built"
    n = torch.cuda.device_count()
    if n < world:
        return False, "fewer visible GPUs than ranks"
    for q in range(n):
        if q != device.index and not torch.cuda.can_device_access_peer(device.index, q):
            return False, f"no peer access from GPU {device.index} to GPU {q}"
    return True, ""


def dma_plan(buckets, shards, pers, world: int, rank: int):
    """Ranges of the copy-engine overlap (stages 1-2: rank q owns flat
    elements [q * S, (q + 1) * S) of each group).

    ``buckets[k]`` lists ``(group, lo, hi)`` arena ranges.  Returns
    ``(sends, covered, remaining)``: ``sends[k]`` lists ``(group, q, e0,
    e1)``, the part of bucket k that this rank copies to peer q; ``covered``
    maps each group to the merged parts of this rank's own shard that the
    buckets bring in, cut to ``pers[group]``-element (16-byte) boundaries;
    ``remaining`` to the rest of the shard, reduced from the peers' arenas at
    the step."""
    sends, mine = [], {i: [] for i in range(len(shards))}
    for ranges in buckets:
        out = []
        for (i, lo, hi) in ranges:
            S = shards[i]
            for q in range(world):
                e0, e1 = max(lo, q * S), min(hi, (q + 1) * S)
                if e1 <= e0:
                    continue
                if q == rank:
                    mine[i].append((e0, e1))
                else:
                    out.append((i, q, e0, e1))
        sends.append(out)
    covered, remaining = {}, {}
    for i, S in enumerate(shards):
        a, b = rank * S, (rank + 1) * S
        per = pers[i]
        merged = []
        for s0, e0 in sorted(mine[i]):
            if merged and s0 <= merged[-1][1]:
                merged[-1] = (merged[-1][0], max(merged[-1][1], e0))
            else:
                merged.append((s0, e0))
        cut = [(-(-s0 // per) * per, e0 // per * per) for s0, e0 in merged]
        covered[i] = [(s0, e0) for s0, e0 in cut if e0 > s0]
        rest, pos = [], a
        for s0, e0 in covered[i]:
            if s0 > pos:
                rest.append((pos, s0))
            pos = max(pos, e0)
        if pos < b:
            rest.append((pos, b))
        remaining[i] = rest
    return sends, covered, remaining


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
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        # epochs of the barrier-type kernels: a device counter each of them
        # advances, so launches replayed from a CUDA graph stay in step
        self.epoch_dev = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._shard32 = {}
        self._step_open = False
        self.dma = False
        self.recv: Optional[PeerHeap] = None
        # phase marker of the optimizer's step timing (None: timing off)
        self.marker = None

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

    def barrier(self) -> None:
        _ext.get().peer_barrier(self.heap.heaps, self.heap.sync_off, self.rank,
                                self.world_size, self.epoch_dev, self.timeout_s, self.status)

    # ---------------------------------------------- bucketed overlap
    BUCKET_SLOTS = 64   # statistics slots (thread blocks) reserved per bucket
    # thread blocks per bucket reduction: it shares the GPU with the backward
    # kernels still running, so it gets a small grid
    BUCKET_BLOCKS = int(os.environ.get("MINISPEED_BUCKET_BLOCKS", "48"))

    def _shard_range(self, g: FlatParamGroup) -> Tuple[int, int]:
        if self.stage == 0:
            return self.rank * g.shard_size, (self.rank + 1) * g.shard_size
        return g.shard_start, g.shard_end

    # how the buckets reach their owners: "dma" (default) copies each peer's
    # part of a bucket into that peer's receive slot with the copy engines
    # as soon as backward has produced it, and the step reduces local slots;
    # "kernel" runs the fused reduce-scatter kernel per bucket on a second
    # stream (it competes with backward for the SMs)
    OVERLAP_MODE = os.environ.get("MINISPEED_OVERLAP_MODE", "dma")

    def plan_buckets(self, buckets: List[List[Tuple[int, int, int]]]) -> int:
        if self.OVERLAP_MODE == "dma" and self.stage in (1, 2):
            return self._plan_dma(buckets)
        self.dma = False
        return self._plan_kernel(buckets)

    def _slot_layout(self, g: FlatParamGroup) -> Tuple[int, int]:
        """(elements per receive slot, element size).  A slot holds one source
        rank's copy of an owner's shard, shifted so that every element sits
        at the same address modulo 16 as in the gradient arena."""
        esz = g.grad_arena.element_size()
        return g.shard_size + 16 // esz, esz

    def _plan_dma(self, buckets: List[List[Tuple[int, int, int]]]) -> int:
        """Copy-engine overlap.  Bucket k's part that rank q owns goes, once
        backward has produced the bucket, straight into q's receive slot for
        this rank (one cudaMemcpyAsync per peer, no SMs).  At the step each
        rank reduces the covered part of its shard from its own arena and its
        local slots (the fused statistics kernel over a table of local
        addresses), and the rest (parameters outside the buckets, the
        unaligned edges) from the peers' arenas as before."""
        self.dma = True
        W, me = self.world_size, self.rank
        regions = []
        for i, g in enumerate(self.groups):
            slot, esz = self._slot_layout(g)
            regions.append((f"recv{i}", W * slot * esz))
        self.recv = PeerHeap(self.device, regions, me, W)   # collective
        shards = [g.shard_size for g in self.groups]
        pers = [16 // g.grad_arena.element_size() for g in self.groups]
        sends, self.covered, self.remaining = dma_plan(buckets, shards, pers, W, me)
        self.dma_copies = []
        for bucket in sends:
            dst, src, nbytes = [], [], []
            for (i, q, e0, e1) in bucket:
                g = self.groups[i]
                slot, esz = self._slot_layout(g)
                align = (q * shards[i]) // pers[i] * pers[i]
                # the copy writes peer memory: it must stay inside q's slot
                # for this rank and read inside this rank's arena (checked
                # once here, not per step)
                if not (q * shards[i] <= e0 < e1 <= min((q + 1) * shards[i], g.numel_padded)
                        and e1 - align <= slot):
                    raise RuntimeError(f"copy-engine plan: group {i} range [{e0}, {e1}) "
                                       f"leaves rank {q}'s receive slot")
                base = self.recv.ptrs[q] + self.recv.offsets[f"recv{i}"] + me * slot * esz
                dst.append(base + (e0 - align) * esz)
                src.append(self.heap.ptrs[me] + self.heap.offsets[f"grad{i}"] + e0 * esz)
                nbytes.append((e1 - e0) * esz)
            self.dma_copies.append((dst, src, nbytes))
        self.recv_tab = {}
        for i, g in enumerate(self.groups):
            slot, esz = self._slot_layout(g)
            # local source table: this rank's arena, and for every peer its
            # slot here, offset so that table[q] + grad_off + e * esz is the
            # address of element e of this rank's shard
            align = (me * shards[i]) // pers[i] * pers[i]
            mine = self.recv.ptrs[me] + self.recv.offsets[f"recv{i}"]
            goff = self.heap.offsets[f"grad{i}"]
            tab = [self.heap.ptrs[me] if q == me else
                   mine + q * slot * esz - goff - align * esz for q in range(W)]
            self.recv_tab[i] = torch.tensor(tab, dtype=torch.int64, device=self.device)
        return 0

    def _plan_kernel(self, buckets: List[List[Tuple[int, int, int]]]) -> int:
        """Fix the reduction of gradient buckets that become final during
        backward.  ``buckets[k]`` lists ``(group, lo, hi)`` arena ranges.  Each
        rank reduces ``[lo, hi)`` cut to its shard and to 8-element (16-byte)
        boundaries; what the buckets leave (other parameters, unaligned
        edges) is reduced at the step.  Returns the statistics slots the
        buckets occupy (bucket k writes slots ``[k*64, (k+1)*64)``)."""
        self.bucket_plan = []
        covered = {i: [] for i in range(len(self.groups))}
        for ranges in buckets:
            segs = []
            for (i, lo, hi) in ranges:
                a, b = self._shard_range(self.groups[i])
                s0, e0 = max(lo, a), min(hi, b)
                s0, e0 = (s0 + 7) // 8 * 8, e0 // 8 * 8
                if e0 > s0:
                    segs.append((i, s0, e0))
                    covered[i].append((s0, e0))
            self.bucket_plan.append(segs)
        self.remaining = {}
        for i, g in enumerate(self.groups):
            a, b = self._shard_range(g)
            rest, cur = [], a
            for s0, e0 in sorted(covered[i]):
                if s0 > cur:
                    rest.append((cur, s0))
                cur = max(cur, e0)
            if cur < b:
                rest.append((cur, b))
            self.remaining[i] = rest
        return len(buckets) * self.BUCKET_SLOTS

    def _out_slice(self, i: int, g: FlatParamGroup, s0: int, e0: int) -> torch.Tensor:
        if self.stage == 0:
            return g._grad[s0:e0]
        a = g.shard_start
        return self._shard_out(i, g)[s0 - a:e0 - a]

    def _reduce_segment(self, i: int, s0: int, e0: int, mul: float, mul_dev, stats,
                        slot: int, max_blocks: int, threads: int = 256, table=None) -> int:
        g = self.groups[i]
        out = self._out_slice(i, g, s0, e0)
        esz = g.grad_arena.element_size()
        aligned = (s0 * esz) % 16 == 0 and (self.heap.offsets[f"grad{i}"] % 16) == 0
        fan = self.heap.offsets[f"grad32_{i}"] if self.stage == 0 else -1
        heaps = self.heap.heaps if table is None else table
        return int(_ext.get().rs_stats(heaps, self.heap.offsets[f"grad{i}"],
                                       DTYPE_CODE[g.grad_arena.dtype], s0, out, self.world_size,
                                       mul, mul_dev, fan, stats.partials, stats.flags, slot,
                                       max_blocks, aligned, threads))

    def launch_bucket(self, k: int, mul_dev: torch.Tensor, stats) -> None:
        """Copy mode: bucket k's parts to their owners' receive slots (copy
        engines, current stream).  Kernel mode: barrier (every rank has this
        bucket's gradients), then the reduction of this rank's part of bucket
        k, on the current stream; the multiplier 1 / loss scale is read from
        ``mul_dev``."""
        if self.dma:
            dst, src, nbytes = self.dma_copies[k]
            _ext.get().copy_many(self.status, dst, src, nbytes)
            return
        self.barrier()
        slot = k * self.BUCKET_SLOTS
        end = slot + self.BUCKET_SLOTS
        for (i, s0, e0) in self.bucket_plan[k]:
            slot += self._reduce_segment(i, s0, e0, 1.0 / self.world_size, mul_dev, stats, slot,
                                         max(1, min(self.BUCKET_BLOCKS, end - slot)), threads=128)

    # ------------------------------------------------------------- step
    def _shard_out(self, i: int, g: FlatParamGroup) -> torch.Tensor:
        if self.stage >= 2:
            return g.grad_shard
        buf = self._shard32.get(i)
        if buf is None:
            buf = self._shard32[i] = torch.zeros(g.shard_size, dtype=torch.float32,
                                                 device=self.device)
        return buf

    def reduce_grads(self, g: FlatParamGroup, arena: torch.Tensor, inv_scale: float, stats=None,
                     overlapped: bool = False):
        i = self.groups.index(g)
        if not self._step_open:
            self.barrier()          # every rank's gradient arena is final
            self._step_open = True
            if self.marker is not None:
                self.marker("barrier")
        if g.grad_arena is not arena:
            raise RuntimeError("gradient arena left the peer heap")
        if overlapped and self.dma:
            # the peers' parts of the buckets are in the local slots (their
            # copies completed before they reached the barrier above)
            tab = self.recv_tab[i]
            for s0, e0 in self.covered[i]:
                left = stats.partials.numel() - stats.used
                stats.used += self._reduce_segment(i, s0, e0, inv_scale / self.world_size, None,
                                                   stats, stats.used, min(left, 148 * 8),
                                                   table=tab)
        if overlapped:
            # the buckets were reduced during backward (or sit in the local
            # slots): the rest comes from the peers' arenas
            for s0, e0 in self.remaining[i]:
                left = stats.partials.numel() - stats.used
                stats.used += self._reduce_segment(i, s0, e0, inv_scale / self.world_size, None,
                                                   stats, stats.used, min(left, 148 * 8))
            if self.stage == 0:
                return g._grad, 1.0, True
            return self._shard_out(i, g), 1.0, True
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
                                 inv_scale / self.world_size, None, fan, stats.partials,
                                 stats.flags, stats.used, min(left, 148 * 8), aligned, 256)
        stats.used += int(nb)
        if self.marker is not None:
            self.marker("rs_stats")
        if self.stage == 0:
            return g._grad, 1.0, True
        return out, 1.0, True

    def stats_need_allreduce(self, stage: int) -> bool:
        return True

    def all_reduce_stats(self, out: torch.Tensor, max_norm: Optional[float] = None) -> None:
        _ext.get().stats_exchange(self.heap.heaps, self.heap.sync_off, self.rank,
                                  self.world_size, self.epoch_dev, out,
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

    def gather_range(self, g: FlatParamGroup, lo: int, hi: int) -> None:
        """Stage 3: arena elements [lo, hi) from their owners' shards (peer
        loads over NVLink), on the current stream."""
        i = self.groups.index(g)
        _ext.get().gather_range(self.heap.heaps, self.heap.offsets[f"pshard{i}"], g.shard_size,
                                lo, hi, g.param_arena)

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
        if self.recv is not None:
            self.recv.close()
            self.recv = None
