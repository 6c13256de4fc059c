"""The training engine: ``initialize`` and :class:`DeepSpeedEngine`.

Public behaviour follows the reference engine (``minispeed/engine.py``):

* ``initialize(model, model_parameters, config)`` returns the engine, which
  also unpacks as ``engine, optimizer, _, lr_scheduler`` (``engine.py:221-224,
  372-389``);
* init order: config -> device -> ``model.to`` -> rank-0 broadcast -> flat
  groups -> fp32 master snapshot -> cast params to the training dtype ->
  (stage 3) partition -> optimizer -> scheduler -> loss scaler
  (``engine.py:90-155``);
* ``backward`` scales the loss by ``loss_scale / gas`` (the ``/gas`` only when
  ``scale_wrt_gas`` and gas > 1) and counts micro-steps (``engine.py:227-251``);
* ``step`` acts only at a not-yet-consumed accumulation boundary and returns
  whether an update was applied; an inf/nan step halves the loss scale, is
  counted in ``skipped_steps``, and does not step the scheduler
  (``engine.py:254-322``).

The optimizer step itself is the device pipeline of
:meth:`minispeed_b200.zero.ZeROOptimizer.boundary_step` (one host
synchronization per step instead of three, one fused kernel per stage of
work).  Device-side phase timers (CUDA events) complement the wall-clock
``engine.timers``.
"""

from __future__ import annotations

import logging
from contextlib import contextmanager, nullcontext
from typing import Iterator, List, Optional

import torch
from torch import nn

from . import checkpoint as ckpt
from . import comm
from .config import DeepSpeedConfig, load_config
from .flat import FlatParamGroup, build_flat_groups
from .ops import _ext
from .ops.nn import batched_colsums, expected_loss_grad
from .optim import build_scheduler
from .precision import DynamicLossScaler
from .utils import DeviceTimers, Timers
from .zero import build_zero_optimizer, make_collectives

logger = logging.getLogger("minispeed_b200")


def _normalize_param_groups(model: nn.Module, model_parameters, defaults: dict) -> List[dict]:
    """torch.optim-style groups from None, an iterable of params, a dict or a
    list of group dicts; config optimizer params are the group defaults
    (reference ``engine.py:44-78``)."""
    if model_parameters is None:
        raw = [list(model.parameters())]
    elif isinstance(model_parameters, dict):
        raw = [model_parameters]
    else:
        items = list(model_parameters)
        raw = items if items and isinstance(items[0], dict) else [items]
    groups = []
    for grp in raw:
        if isinstance(grp, dict):
            params, opts = grp.get("params", []), {k: v for k, v in grp.items() if k != "params"}
        else:
            params, opts = grp, {}
        if isinstance(params, torch.Tensor):
            params = [params]
        merged = dict(defaults)
        merged.update(opts)
        merged["params"] = [p for p in params if isinstance(p, nn.Parameter) and p.requires_grad]
        if merged["params"]:
            groups.append(merged)
    if not groups:
        raise ValueError("No trainable parameters found")
    return groups


class DeepSpeedEngine:
    """Wraps an ``nn.Module`` with ZeRO data parallelism and mixed precision."""

    def __init__(self, model: nn.Module, config, model_parameters=None):
        self.config: DeepSpeedConfig = load_config(config, world_size=comm.get_world_size())
        self.rank = comm.get_rank()
        self.world_size = comm.get_world_size()
        self.device = comm.resolve_device()
        if self.device.type == "cuda":
            if self.device.index is None:
                # MINISPEED_DEVICE=cuda: the current device (as the reference,
                # which uses the bare "cuda" device)
                self.device = torch.device("cuda", torch.cuda.current_device())
            torch.cuda.set_device(self.device)
        self.timers = Timers()
        # CUDA-event times of the same phases plus "forward" (b200.device_timers)
        self.device_timers = DeviceTimers()
        self._device_timing = self.config.b200.device_timers and self.device.type == "cuda"
        self.module = model.to(self.device)
        self._broadcast_model()

        groups = _normalize_param_groups(model, model_parameters, self.config.optimizer_params)
        self.flat_groups: List[FlatParamGroup]
        self.flat_groups, option_groups = build_flat_groups(
            groups, rank=self.rank, world_size=self.world_size,
            zero_stage=self.config.zero_stage, device=self.device)
        for g in self.flat_groups:
            g.copy_model_to_flat()  # params are still in their original dtype here

        self._param_dtype = None
        if self.config.dtype != "fp32":
            self._param_dtype = self.config.torch_dtype
            for g in self.flat_groups:
                g.cast_params(self._param_dtype)
        if self.config.zero_stage >= 3:
            for g in self.flat_groups:
                g.partition_params()

        coll = make_collectives(self.world_size, self.rank, self.device,
                                self.config.b200.comm, self.config.b200)
        self.optimizer = build_zero_optimizer(self.flat_groups, option_groups,
                                              zero_stage=self.config.zero_stage,
                                              collectives=coll)
        self.lr_scheduler = build_scheduler(self.optimizer, self.config.scheduler_type,
                                            self.config.scheduler_params)
        fp16 = self.config.fp16_enabled
        self.loss_scaler = DynamicLossScaler(enabled=fp16, init_scale=self.config.loss_scale,
                                             scale_window=self.config.loss_scale_window)
        if fp16 and self.config.loss_scale == 0:
            self.loss_scaler.set_scale_from_power(self.config.initial_scale_power)

        self.micro_steps = 0
        self.global_steps = 0
        self.skipped_steps = 0
        self._consumed_boundary = -1
        self.grad_norm: Optional[float] = None
        self._window_open = False
        # captured micro-steps of train_batch (CUDA graphs), one per signature:
        # with gradient accumulation and overlap, the window's last micro-step
        # (which launches the bucket transfers) differs from the others
        self._graphs = {}
        self._graph = None          # the graph replayed last
        self._graph_eager = {}      # eager micro-steps run per signature
        # the bounds-checked debug build: its device records are read (and a
        # failure raised) after every step
        self._debug_bounds = self.device.type == "cuda" and _ext.debug_build()
        self._overlap_now = False   # this micro-step's backward reduces buckets
        self._bucket_hooks = self._setup_overlap() + self._setup_layer_gather()

    # ----------------------------------------------------------- properties
    @property
    def gas(self) -> int:
        return self.config.gas

    @property
    def is_gradient_accumulation_boundary(self) -> bool:
        return self.micro_steps > 0 and self.micro_steps % self.gas == 0

    @property
    def _boundary_pending(self) -> bool:
        return self.is_gradient_accumulation_boundary and self._consumed_boundary != self.micro_steps

    @property
    def loss_scale(self) -> float:
        return self.loss_scaler.loss_scale_factor

    @property
    def parameters(self):
        return self.module.parameters()

    @property
    def collectives(self) -> str:
        """Name of the gradient/parameter communication strategy in use."""
        return self.optimizer.coll.name

    # --------------------------------------------------------- nn surface
    def _cast_inputs(self, obj):
        """Cast floating-point inputs to the model dtype, recursively
        (reference ``engine.py:182-198``)."""
        dt = self._param_dtype
        if dt is None:
            return obj
        if isinstance(obj, torch.Tensor):
            return obj.to(dt) if obj.is_floating_point() and obj.dtype != dt else obj
        if isinstance(obj, dict):
            return {k: self._cast_inputs(v) for k, v in obj.items()}
        if isinstance(obj, tuple):
            return tuple(self._cast_inputs(v) for v in obj)
        if isinstance(obj, list):
            return [self._cast_inputs(v) for v in obj]
        return obj

    def _open_window(self) -> None:
        """First forward of an accumulation window: bind the gradient arenas
        so autograd accumulates straight into them."""
        if self._window_open or not torch.is_grad_enabled() or not self.module.training:
            return
        for g in self.flat_groups:
            if g.params_materialized:
                g.rebind()
                g.ensure_grad_arena()
        self._window_open = True

    # ---------------------------------------------- overlapped reductions
    def _bucket_modules(self) -> List[nn.Module]:
        fn = getattr(self.module, "bucket_modules", None)
        if callable(fn):
            return list(fn())
        for name in ("blocks", "layers", "h"):
            mods = getattr(self.module, name, None)
            if isinstance(mods, nn.ModuleList) and len(mods) > 0:
                return list(mods)
        return []

    def _setup_overlap(self) -> list:
        """Reduce each block's gradients while backward continues with the
        blocks before it (fused collectives, ``b200.overlap``).  A marker
        wraps the block's input; its backward runs once the block's whole
        backward has written the block's gradients."""
        if not (self.config.b200.overlap and self.world_size > 1 and self.device.type == "cuda"):
            return []
        mods = self._bucket_modules()
        if not mods or not self.optimizer.plan_overlap([list(m.parameters()) for m in mods]):
            return []
        hooks = []
        for k, m in enumerate(mods):
            hooks.append(m.register_forward_pre_hook(self._bucket_hook(k)))
        return hooks

    def _setup_layer_gather(self) -> list:
        """Stage 3 with fused collectives: gather each block's parameters one
        block ahead of its forward (``ZeROStage3Optimizer.layer_ready``)."""
        plan = getattr(self.optimizer, "plan_layer_gather", None)
        if plan is None or self.world_size <= 1 or self.device.type != "cuda":
            return []
        mods = self._bucket_modules()
        if not mods or not plan([list(m.parameters()) for m in mods]):
            return []
        hooks = []
        for k, m in enumerate(mods):
            hooks.append(m.register_forward_pre_hook(
                lambda module, args, k=k: self.optimizer.layer_ready(k)))
        return hooks

    def _bucket_hook(self, k: int):
        def hook(module, args):
            if (not self._overlap_now or not torch.is_grad_enabled() or not args
                    or not isinstance(args[0], torch.Tensor) or not args[0].requires_grad):
                return None
            return (_BucketMark.apply(args[0], self.optimizer, k),) + tuple(args[1:])
        return hook

    def _begin_micro_step(self) -> None:
        """Decided at forward time: the micro-step that closes an accumulation
        window reduces its buckets during backward."""
        self._overlap_now = bool(self._bucket_hooks) and self.module.training and \
            (self.micro_steps + 1) % self.gas == 0
        if self._overlap_now:
            self.optimizer.set_loss_scale(self.loss_scaler.loss_scale_factor)

    def forward(self, *args, **kwargs):
        """Run the module on inputs cast to the training dtype (stage 3: gathering
        the parameters first) and open the micro-step's gradient window."""
        if not self.optimizer.params_gathered:
            with self._phase("gather"):
                if getattr(self.optimizer, "plan_layer_gather", None) is not None:
                    self.optimizer.gather_parameters(layerwise=True)
                else:
                    self.optimizer.gather_parameters()
        self._open_window()
        self._begin_micro_step()
        with self._device_phase("forward"), expected_loss_grad(self._loss_grad_hint()):
            return self.module(*self._cast_inputs(args), **self._cast_inputs(kwargs))

    def _loss_grad_hint(self) -> Optional[torch.Tensor]:
        """The upstream gradient :meth:`backward` will give the module's loss
        (loss scale / gradient-accumulation steps), as a device scalar: the
        fused cross-entropy computes its gradient in the forward for it."""
        if self.device.type != "cuda" or not self.module.training:
            return None
        factor = self.loss_scaler.loss_scale_factor
        if self.gas > 1:
            factor /= self.gas
        if getattr(self, "_hint_dev", None) is None:
            self._hint_dev = torch.empty(1, dtype=torch.float32, device=self.device)
            self._hint_val = None
        if self._hint_val != factor:
            self._hint_dev.fill_(factor)
            self._hint_val = factor
        return self._hint_dev

    @contextmanager
    def _phase(self, name: str):
        """Wall-clock section of ``engine.timers`` (and of ``device_timers``
        when ``b200.device_timers`` is on)."""
        with self.timers.timer(name), self._device_phase(name):
            yield

    def _device_phase(self, name: str):
        return self.device_timers.timer(name) if self._device_timing else nullcontext()

    def device_time_ms(self) -> dict:
        """Milliseconds of GPU time per phase (``forward``, ``backward``,
        ``step``, ``reduce``, ``gather``) since the last reset, from CUDA
        events on the launching stream; empty unless ``b200.device_timers``
        is on.  Synchronizes the GPU."""
        return self.device_timers.elapsed_ms() if self._device_timing else {}

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def train(self, mode: bool = True):
        self.module.train(mode)
        return self

    def eval(self):
        self.module.eval()
        return self

    def __iter__(self) -> Iterator:
        return iter((self, self.optimizer, None, self.lr_scheduler))

    # ------------------------------------------------------------ backward
    def _scale_loss(self, loss: torch.Tensor, scale_wrt_gas: bool) -> torch.Tensor:
        factor = self.loss_scaler.loss_scale_factor
        if scale_wrt_gas and self.gas > 1:
            factor /= self.gas
        return loss if factor == 1.0 else loss * factor

    def backward(self, loss: torch.Tensor, scale_wrt_gas: bool = True,
                 retain_graph: bool = False, create_graph: bool = False) -> None:
        # bias and norm-weight gradient finishes run batched (ops.nn)
        with self._phase("backward"), batched_colsums():
            self._scale_loss(loss, scale_wrt_gas).backward(retain_graph=retain_graph,
                                                           create_graph=create_graph)
        self.micro_steps += 1

    # --------------------------------------------------------- train_batch
    def train_batch(self, *args, **kwargs) -> torch.Tensor:
        """One micro-step: ``loss = module(*args, **kwargs)`` (the module
        returns a scalar loss), the scaled backward, then :meth:`step` (which
        acts only at an accumulation boundary).  Returns the loss.

        With ``b200.cuda_graph`` on a CUDA device at ZeRO stage 0-2, the
        forward + backward of a given input signature is captured once, after
        ``b200.graph_warmup`` eager micro-steps, and replayed from then on
        (:mod:`minispeed_b200.graphs`).  Input tensors may live on the host;
        they are copied into the graph's static inputs.  The returned loss
        tensor is then the graph's output, overwritten by the next call.
        """
        if self._graph_usable():
            loss = self._graph_micro_step(args, kwargs)
        else:
            loss = self.forward(*self._to_device(args), **self._to_device(kwargs))
            self.backward(loss)
        self.step()
        # detached: a caller holding the loss keeps no autograd graph alive
        # (a live graph would pin its AccumulateGrad nodes to the stream of
        # that step and break a later capture)
        return loss.detach()

    def _to_device(self, obj):
        if isinstance(obj, torch.Tensor):
            return obj.to(self.device, non_blocking=True)
        if isinstance(obj, dict):
            return {k: self._to_device(v) for k, v in obj.items()}
        if isinstance(obj, (list, tuple)):
            return type(obj)(self._to_device(v) for v in obj)
        return obj

    def _graph_usable(self) -> bool:
        return (self.config.b200.cuda_graph and self.device.type == "cuda"
                and self.config.zero_stage < 3 and self.module.training
                and torch.is_grad_enabled())

    def _graph_micro_step(self, args, kwargs) -> torch.Tensor:
        from .graphs import MicroStepGraph, signature
        self._begin_micro_step()
        sig, _ = signature(args, kwargs)
        sig = (sig, self._overlap_now)
        st = self._graphs.get(sig)
        if st is not None and st.graph is not None and not st.valid():
            st.release()
            del self._graphs[sig]
            st = None
        if st is None:
            side = self._graph_stream()
            cur = torch.cuda.current_stream(self.device)
            side.wait_stream(cur)
            n = self._graph_eager.get(sig, 0)
            if n < self.config.b200.graph_warmup:
                # eager micro-steps first (GEMM autotuning, lazy library
                # state), on the stream the capture will use
                self._graph_eager[sig] = n + 1
                with torch.cuda.stream(side):
                    loss = self.forward(*self._to_device(args), **self._to_device(kwargs))
                    self.backward(loss)
                cur.wait_stream(side)
                return loss
            if len(self._graphs) >= self.MAX_GRAPHS:
                # the signature replayed longest ago goes (inputs of new shapes)
                old = next(iter(self._graphs))
                self._graphs.pop(old).release()
            torch.cuda.empty_cache()
            st = MicroStepGraph(self, args, kwargs)
            st.sig = sig            # inputs and whether the bucket reductions are captured
            st.capture(side)
            cur.wait_stream(side)
            self._graphs[sig] = st
        else:
            self._graphs[sig] = self._graphs.pop(sig)   # most recently used last
        self._graph = st
        factor = self.loss_scaler.loss_scale_factor
        if self.gas > 1:
            factor /= self.gas
        st.set_seed(factor)
        st.load_inputs(args, kwargs)
        if not self._window_open:
            # the graph checked the arena addresses; only the p.grad views
            # (which the step reads) need to be in place
            for g in self.flat_groups:
                g.ensure_grad_arena()
            self._window_open = True
        with self._phase("backward"):
            loss = st.replay()
        if st.overlap:
            self.optimizer._overlap_ran = True   # the replay ran the bucket reductions
        self.micro_steps += 1
        return loss

    def _graph_stream(self) -> torch.cuda.Stream:
        if getattr(self, "_side_stream", None) is None:
            self._side_stream = torch.cuda.Stream(self.device)
        return self._side_stream

    MAX_GRAPHS = 4      # captured micro-step signatures kept at once

    def release_graphs(self) -> None:
        """Drop the captured micro-step graphs and their memory pools."""
        for st in self._graphs.values():
            st.release()
        self._graphs = {}
        self._graph = None
        self._graph_eager = {}

    # ---------------------------------------------------------------- step
    def step(self) -> bool:
        """Apply the optimizer at a pending accumulation boundary.

        Returns True only when an update was applied."""
        if not self._boundary_pending:
            return False
        self._consumed_boundary = self.micro_steps
        with self._phase("step"):
            applied = self._take_optimizer_step()
        if self._debug_bounds:
            _ext.check_bounds()
        return applied

    @torch.no_grad()
    def _take_optimizer_step(self) -> bool:
        scale = self.loss_scaler.loss_scale_factor
        with self._phase("reduce"):
            applied, norm = self.optimizer.boundary_step(scale, self.config.gradient_clipping)
        self.optimizer.after_step(applied)
        self._window_open = False
        if not applied:
            self.loss_scaler.update(overflow=True)
            self.skipped_steps += 1
            self.optimizer.zero_grad()
            if self.skipped_steps % max(1, self.config.steps_per_print) == 0:
                logger.warning("rank %d: inf/nan gradients at micro_step=%d, step skipped "
                               "(loss_scale=%.1f, skipped=%d)", self.rank, self.micro_steps,
                               self.loss_scaler.scale, self.skipped_steps)
            return False
        self.grad_norm = norm
        self.loss_scaler.update(overflow=False)
        self.lr_scheduler.step()
        self.optimizer.zero_grad()
        self.global_steps += 1
        return True

    def zero_grad(self, set_to_none: bool = True) -> None:
        for g in self.flat_groups:
            g.zero_grad()
        for p in self.module.parameters():
            p.grad = None
        self._window_open = False

    # ------------------------------------------------------- checkpointing
    def save_checkpoint(self, save_dir: str, tag: Optional[str] = None, **kwargs):
        return ckpt.save_checkpoint(self, save_dir, tag=tag, **kwargs)

    def load_checkpoint(self, load_dir: str, tag: Optional[str] = None, **kwargs):
        return ckpt.load_checkpoint(self, load_dir, tag=tag, **kwargs)

    def state_dict(self):
        self.optimizer.gather_parameters()
        return self.module.state_dict()

    def load_state_dict(self, state_dict):
        self.optimizer.gather_parameters()
        self.module.load_state_dict(state_dict)
        for g in self.flat_groups:
            g.copy_model_to_flat()

    # -------------------------------------------------------------- helpers
    @torch.no_grad()
    def _broadcast_model(self) -> None:
        if not comm.is_distributed():
            return
        tensors = [p.data for p in self.module.parameters()]
        tensors += [b.data for b in self.module.buffers()]
        comm.broadcast_tensors(tensors, src=0)

    def get_loss_scale(self) -> float:
        return self.loss_scaler.scale

    def get_gradient_norm(self) -> Optional[float]:
        return self.grad_norm

    def close(self) -> None:
        """Release communication resources (peer mappings, buffers)."""
        self.release_graphs()
        for h in self._bucket_hooks:
            h.remove()
        self._bucket_hooks = []
        self.optimizer.close()

    def __repr__(self) -> str:  # pragma: no cover
        return (f"DeepSpeedEngine({self.config!r}, global_steps={self.global_steps}, "
                f"micro_steps={self.micro_steps})")


class _BucketMark(torch.autograd.Function):
    """Identity on a block's input; its backward launches the reduction of
    the block's gradient bucket."""

    @staticmethod
    def forward(ctx, x, optimizer, k):
        ctx.optimizer = optimizer
        ctx.k = k
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        ctx.optimizer.launch_bucket(ctx.k)
        return grad, None, None


def initialize(model: Optional[nn.Module] = None, model_parameters=None, config=None,
               model_args=None):
    """Initialize distributed state and build the engine.

    ``engine, optimizer, _, lr_scheduler = initialize(...)`` also works."""
    if model is None:
        raise ValueError("model is required")
    comm.init_distributed()
    engine = DeepSpeedEngine(model, config, model_parameters=model_parameters)
    if comm.get_rank() == 0:
        logger.info("minispeed_b200 initialized: %s (collectives=%s)", engine.config,
                    engine.collectives)
    return engine
