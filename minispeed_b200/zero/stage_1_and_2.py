"""ZeRO stages 0, 1 and 2 and the B200 optimizer-step pipeline.

Stage semantics (reference ``minispeed/zero/stage_1_and_2.py:1-155``):

=======  ==========================================================
stage 0  gradients all-reduced; full optimizer state on every rank
stage 1  optimizer state partitioned; updated shards all-gathered
stage 2  gradients reduce-scattered as well
=======  ==========================================================

The pipeline (:meth:`ZeROOptimizer.boundary_step`) replaces the reference's
flatten -> isfinite (host sync) -> flag all-reduce (host sync) -> unscale ->
reduce -> sum of squares (host sync) -> clip -> ~10-kernel Adam -> fp32
all-gather -> per-param copies chain with:

1. ``reduce_grads`` per group (a strategy from :mod:`..parallel`): nothing at
   world size 1 (the model-dtype gradient arena is read in place), a fused
   NVLink reduce-scatter/all-reduce kernel, or NCCL;
2. the fused statistics kernel over the reduced gradient (flag + sum of
   squares into device scratch), folded on the device into
   ``[flag, sumsq, norm, clip_coef]`` (summed over ranks where the gradient
   is sharded: the norm is the exact global norm at every stage, including
   stage 1, where the reference only sums this rank's shard);
3. one fused AdamW kernel per group that skips itself on overflow, applies
   unscale * clip on the fly and writes the cast parameters;
4. the parameter all-gather (stages 1-2);
5. ONE device-to-host read of ``[flag, norm]`` at the very end.

The reference-granular methods (``reduce_gradients``, ``clip_gradients``,
``step``, ``sync_parameters``) remain for callers that drive the steps
themselves; they follow the reference's library-collective sequence.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from .. import comm
from ..flat import FlatParamGroup
from ..ops import kernels
from ..ops.nn import flush_colsums
from ..optim.adam import FlatAdam
from ..parallel.collectives import LibraryCollectives, LocalCollectives


def make_collectives(world_size: int, rank: int, device: torch.device, mode: str = "auto",
                     options=None):
    """Pick the reduction/gather strategy for this process."""
    if world_size <= 1:
        return LocalCollectives()
    if mode in ("auto", "fused") and device.type == "cuda":
        from ..parallel import fused

        ok, why = fused.supported(device)
        if ok:
            return fused.FusedCollectives(world_size, rank, device, options)
        if mode == "fused":
            raise RuntimeError(f"b200.comm=fused requested but unavailable: {why}")
    return LibraryCollectives(world_size, rank)


class ZeROOptimizer:
    def __init__(self, flat_groups: List[FlatParamGroup], option_groups: List[dict],
                 zero_stage: int = 0, collectives=None):
        if zero_stage not in (0, 1, 2, 3):
            raise ValueError(f"Unsupported ZeRO stage: {zero_stage}")
        self.flat_groups = flat_groups
        self.zero_stage = zero_stage
        self.world_size = comm.get_world_size()
        self.rank = comm.get_rank()
        self.adam = FlatAdam(flat_groups, option_groups, zero_stage=zero_stage)
        self.grad_norm: Optional[float] = None
        device = flat_groups[0].device
        self.coll = collectives if collectives is not None else make_collectives(
            self.world_size, self.rank, device)
        self.coll.attach(flat_groups, zero_stage)
        self.stats = kernels.StepStats(device)
        self._host_stats = (torch.zeros(4, dtype=torch.float32, pin_memory=True)
                            if device.type == "cuda" else None)
        # stages 1-2 only all-gather the model-dtype params each step; the
        # fp32 masters outside this rank's shard are refreshed on demand
        self._masters_stale = False
        # optional CUDA-event timing of the phases of each step: a list that
        # gets one {phase: ms} dict per step (set it to [] to enable)
        self.phase_log = None
        self._marks = None
        # bucketed reduction overlapped with backward (fused collectives)
        self.overlap_slots = 0
        self._overlap_ran = False
        self.comm_stream = None
        self.inv_scale_dev = None
        self._inv_scale_host = None

    # ------------------------------------------------------ torch surface
    @property
    def param_groups(self) -> List[dict]:
        return self.adam.param_groups

    @property
    def state(self) -> List[dict]:
        return self.adam.state

    def zero_grad(self) -> None:
        for g in self.flat_groups:
            g.zero_grad()

    # ------------------------------------------- overlap with backward
    def plan_overlap(self, buckets: List[List[torch.nn.Parameter]]) -> bool:
        """Set up the reduction of each parameter bucket as soon as backward
        has produced it (``launch_bucket``).  A bucket's parameters must fill
        one contiguous arena range per group.  Returns False (no overlap) when
        the collectives cannot run buckets or a bucket does not qualify."""
        if not hasattr(self.coll, "plan_buckets") or self.stats.device.type != "cuda":
            return False
        where = {}
        for gi, g in enumerate(self.flat_groups):
            for p, off, n in zip(g.params, g._offsets_int, g._numels):
                where[id(p)] = (gi, off, n)
        seen, plan = set(), []
        for params in buckets:
            spans = {}
            for p in params:
                if id(p) not in where or id(p) in seen:
                    return False
                seen.add(id(p))
                gi, off, n = where[id(p)]
                lo, hi, tot = spans.get(gi, (off, off + n, 0))
                spans[gi] = (min(lo, off), max(hi, off + n), tot + n)
            if any(hi - lo != tot for lo, hi, tot in spans.values()):
                return False        # not one contiguous range
            plan.append([(gi, lo, hi) for gi, (lo, hi, _) in sorted(spans.items())])
        if not plan:
            return False
        self.overlap_slots = self.coll.plan_buckets(plan)
        self.comm_stream = torch.cuda.Stream(self.stats.device)
        self.inv_scale_dev = torch.ones(1, dtype=torch.float32, device=self.stats.device)
        return True

    def set_loss_scale(self, scale: float) -> None:
        """The multiplier the overlapped reductions read (1 / loss scale)."""
        if self.inv_scale_dev is not None and scale != self._inv_scale_host:
            self.inv_scale_dev.fill_(1.0 / float(scale))
            self._inv_scale_host = scale

    def launch_bucket(self, k: int) -> None:
        """Reduce bucket k on the communication stream, after the work the
        current (backward) stream has queued so far."""
        flush_colsums()   # the bucket's bias and norm-weight gradients are complete
        cur = torch.cuda.current_stream(self.stats.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            self.coll.launch_bucket(k, self.inv_scale_dev, self.stats)
        self._overlap_ran = True

    def join_comm(self) -> None:
        """Make the current stream wait for the overlapped reductions."""
        if self.comm_stream is not None:
            torch.cuda.current_stream(self.stats.device).wait_stream(self.comm_stream)

    # ---------------------------------------------- parameter lifecycle
    @property
    def params_gathered(self) -> bool:
        return True

    def gather_parameters(self) -> None:
        """Stage-3 hook (no-op: stages 0-2 keep full params resident)."""

    def free_parameters(self, refresh: bool = True) -> None:
        """Stage-3 hook (no-op for stages 0-2)."""

    @torch.no_grad()
    def sync_parameters(self) -> None:
        """Push the fp32 masters into the model params (library path)."""
        for g in self.flat_groups:
            g.copy_flat_to_model()

    @torch.no_grad()
    def sync_master_weights(self) -> None:
        """Make every rank's full fp32 master buffer current (stages 1-2)."""
        if not self._masters_stale:
            return
        for g in self.flat_groups:
            self.coll.gather_masters(g)
        self._masters_stale = False

    # ------------------------------------------------------ the pipeline
    def _param_target(self, g: FlatParamGroup) -> Optional[torch.Tensor]:
        """Where AdamW writes the model-dtype cast of the updated shard."""
        if g._partitioned:
            return g.param_shard
        return g.param_arena[g.shard_start:g.shard_end]

    @torch.no_grad()
    def boundary_step(self, loss_scale: float, max_norm: Optional[float]
                      ) -> Tuple[bool, Optional[float]]:
        """Run the whole optimizer step.  Returns ``(applied, grad_norm)``;
        on overflow nothing was updated on any rank."""
        inv = 1.0 / float(loss_scale)
        st = self.stats
        st.reset()
        overlapped = self._overlap_ran
        self._overlap_ran = False
        if overlapped:
            self.join_comm()
            st.used = self.overlap_slots
        timing = self.phase_log is not None and st.device.type == "cuda"
        self._marks = [] if timing else None
        self.coll.marker = self._mark if timing else None
        self._mark("start")
        grads, mul = [], 1.0
        for g in self.flat_groups:
            arena = g.collect_grads()
            if overlapped:
                red, mul, stats_done = self.coll.reduce_grads(g, arena, inv, st, overlapped=True)
            else:
                red, mul, stats_done = self.coll.reduce_grads(g, arena, inv, st)
            if not stats_done:
                st.accumulate(red, mul)
            grads.append(red)
        self._mark("reduce")
        if self.coll.stats_need_allreduce(self.zero_stage):
            st.finalize(max_norm, epilogue=False)
            self.coll.all_reduce_stats(st.out)
            out = st.epilogue(max_norm)
        else:
            out = st.finalize(max_norm)
        self._mark("stats")
        targets = [self._param_target(g) for g in self.flat_groups]
        fanouts = [self.coll.fanout(g) for g in self.flat_groups]
        self.adam.fused_step(grads, out, mul, max_norm, targets, fanouts)
        self._mark("adamw")
        if 1 <= self.zero_stage <= 2 and self.world_size > 1:
            for g in self.flat_groups:
                self.coll.gather_params(g)
            self._masters_stale = True
        self.coll.end_step()
        self._mark("gather")
        flag, norm = self._read_stats(out)
        self.coll.check()
        if timing:
            self.phase_log.append(self._phase_times())
            self.coll.marker = None
        self._marks = None
        if flag:
            return False, None
        self.adam.commit_step()
        self.grad_norm = norm
        return True, norm

    def _mark(self, name: str) -> None:
        """Record a CUDA event that ends phase ``name`` of this step (timing on)."""
        if self._marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((name, ev))

    def _phase_times(self) -> dict:
        """Milliseconds from each mark to the next, under the later mark's
        name (after the step's one host read, so every event has completed).
        Phases: ``barrier`` (peer barrier: every rank's backward is done),
        ``rs_stats`` (fused reduce-scatter + statistics), ``reduce`` (what
        else the reduction took: library collectives, local statistics),
        ``stats`` (statistics exchange / finalize), ``adamw`` (fused AdamW,
        with the parameter fan-out at stages 1-2), ``gather`` (parameter
        all-gather or the final peer barrier)."""
        out = {}
        for (_, a), (name, b) in zip(self._marks, self._marks[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out

    def _read_stats(self, out: torch.Tensor) -> Tuple[bool, float]:
        if out.is_cuda:
            h = self._host_stats
            h.copy_(out[:4], non_blocking=True)
            torch.cuda.current_stream(out.device).synchronize()
            vals = h.tolist()
        else:
            vals = out[:4].tolist()
        return vals[kernels.OUT_FLAG] != 0.0, float(vals[kernels.OUT_NORM])

    def after_step(self, applied: bool) -> None:
        """Parameter bookkeeping once the step outcome is known."""

    # ------------------------------------- reference-granular library API
    @torch.no_grad()
    def reduce_gradients(self) -> None:
        ws = self.world_size
        for g in self.flat_groups:
            if self.zero_stage >= 2:
                comm.reduce_scatter(g.grad_shard, g.grad)
                if ws > 1:
                    g.grad_shard.div_(ws)
            else:
                comm.all_reduce(g.grad)
                if ws > 1:
                    g.grad.div_(ws)

    @torch.no_grad()
    def clip_gradients(self, max_norm: Optional[float]) -> float:
        """Exact global L2 norm (+ optional clipping) of the reduced grads."""
        total = torch.zeros((), dtype=torch.float32, device=self.flat_groups[0].device)
        for g in self.flat_groups:
            total += g.local_grad_sumsq()
        if self.zero_stage >= 1 and self.world_size > 1:
            comm.all_reduce(total, op="sum")
        norm = float(total.sqrt().item())
        self.grad_norm = norm
        if max_norm is not None and norm > max_norm:
            coef = max_norm / (norm + 1e-6)
            for g in self.flat_groups:
                g.scale_grads(coef)
        return norm

    @torch.no_grad()
    def step(self) -> bool:
        updated = self.adam.step()
        if self.zero_stage >= 1 and self.world_size > 1:
            for g in self.flat_groups:
                full = torch.empty_like(g.data)
                comm.all_gather_flat(full, g.shard)
                g.data.copy_(full)
        return updated

    # --------------------------------------------------------- persistence
    def state_dict(self) -> dict:
        return self.adam.state_dict()

    def load_state_dict(self, state: dict) -> None:
        self.adam.load_state_dict(state)

    def close(self) -> None:
        self.coll.close()
