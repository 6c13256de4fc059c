"""CUDA-graph replay of a training micro-step (forward + scaled backward).

A GPT-2-small micro-step issues about 400 kernels through Python autograd;
on a B200 the host needs longer to issue them than the GPU needs to run
them, so the device idles between kernels.  :class:`MicroStepGraph`
captures the whole forward + backward once and replays it with one launch.

What stays valid across replays:
- parameters and gradients live in the engine's flat arenas, whose
  addresses do not change between steps (the arenas are zeroed in place;
  the recorded addresses are checked before every replay);
- inputs are copied into static device tensors recorded in the graph
  (host tensors, pinned or not, are copied host-to-device directly);
- the backward seed (loss scale / gradient-accumulation factor) is a device
  scalar read by the graph, so dynamic loss scaling needs no recapture;
- activations come from the graph's private memory pool.

The eager warm-up micro-steps and the capture run on one engine-owned side
stream, and ``train_batch`` hands back detached losses: autograd binds each
parameter's gradient accumulator to the stream of the graph that created it,
and one bound to another stream would make the captured backward wait on
uncaptured work.

The optimizer step is not captured: it ends with the host read of the
overflow flag and norm that decides skip / scale / scheduler, and issues
only a handful of fused kernels.

There is no reference counterpart: the reference runs every micro-step
eagerly (``engine.py:200-251``); this is the B200 execution path of the same
forward / backward semantics.
"""

from __future__ import annotations

from typing import Any, List, Optional, Tuple

import torch

from .ops import _ext
from .ops.nn import batched_colsums, expected_loss_grad


def _flatten(obj, out: List[torch.Tensor]):
    """Tensors of a nested args structure in a fixed order; returns the
    structure's signature (shapes, dtypes, non-tensor values)."""
    if isinstance(obj, torch.Tensor):
        out.append(obj)
        return ("T", tuple(obj.shape), obj.dtype)
    if isinstance(obj, (list, tuple)):
        return (type(obj).__name__, tuple(_flatten(v, out) for v in obj))
    if isinstance(obj, dict):
        return ("dict", tuple((k, _flatten(obj[k], out)) for k in sorted(obj)))
    return ("V", obj)


def _rebuild(obj, it):
    if isinstance(obj, torch.Tensor):
        return next(it)
    if isinstance(obj, list):
        return [_rebuild(v, it) for v in obj]
    if isinstance(obj, tuple):
        return tuple(_rebuild(v, it) for v in obj)
    if isinstance(obj, dict):
        return {k: _rebuild(obj[k], it) for k in obj}
    return obj


def signature(args, kwargs) -> Tuple[Any, List[torch.Tensor]]:
    tensors: List[torch.Tensor] = []
    sig = (_flatten(list(args), tensors), _flatten(dict(kwargs), tensors))
    return sig, tensors


class MicroStepGraph:
    """One captured forward + backward for one input signature."""

    def __init__(self, engine, args, kwargs):
        self.engine = engine
        self.device = engine.device
        self.sig, tensors = signature(args, kwargs)
        self.static = [torch.empty(t.shape, dtype=t.dtype, device=self.device) for t in tensors]
        it = iter(self.static)
        self.args = _rebuild(list(args), it)
        self.kwargs = _rebuild(dict(kwargs), it)
        self.seed = torch.ones((), dtype=torch.float32, device=self.device)
        self._seed_value = 1.0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.loss: Optional[torch.Tensor] = None
        self.overlap = engine._overlap_now   # captured with the bucket reductions
        self.kernels = 0          # this library's kernels per replay
        self.replays = 0
        self._ptrs: Tuple[int, ...] = ()

    def _arena_ptrs(self) -> Tuple[int, ...]:
        ptrs = []
        for g in self.engine.flat_groups:
            for t in (g.param_arena, g.grad_arena):
                ptrs.append(t.data_ptr() if t is not None else 0)
        return tuple(ptrs)

    def valid(self) -> bool:
        return self.graph is not None and self._ptrs == self._arena_ptrs()

    def load_inputs(self, args, kwargs) -> None:
        _, tensors = signature(args, kwargs)
        for dst, src in zip(self.static, tensors):
            dst.copy_(src, non_blocking=True)

    def set_seed(self, value: float) -> None:
        if value != self._seed_value:
            self.seed.fill_(value)
            self._seed_value = value

    def capture(self, stream: torch.cuda.Stream) -> None:
        """Record forward + backward on ``stream`` (the stream the eager
        warm-up micro-steps ran on)."""
        eng = self.engine
        eng._open_window()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        n0 = _ext.launch_count()
        with torch.cuda.graph(g, stream=stream):
            # the fused cross-entropy computes its gradient for this seed
            with expected_loss_grad(self.seed):
                loss = eng.module(*eng._cast_inputs(self.args), **eng._cast_inputs(self.kwargs))
            if not isinstance(loss, torch.Tensor) or loss.dim() != 0:
                raise RuntimeError("train_batch: the module must return a scalar loss")
            with batched_colsums():
                torch.autograd.backward(loss, self.seed.to(loss.dtype))
            if self.overlap:
                eng.optimizer.join_comm()   # the bucket reductions rejoin the graph
        if self.overlap:
            eng.optimizer._overlap_ran = False   # captured, not run
        self.kernels = _ext.launch_count() - n0
        self.graph = g
        self.loss = loss.detach()    # the graph's output buffer, no autograd refs
        self._ptrs = self._arena_ptrs()

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        self.replays += 1
        if self.kernels:
            _ext.get().count_launches(self.kernels)
        return self.loss

    def release(self) -> None:
        self.graph = None
        self.loss = None
        self.static = []
