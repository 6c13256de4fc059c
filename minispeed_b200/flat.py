"""Flat parameter groups: one contiguous arena per parameter group.

Layout (must stay identical to the reference for checkpoint compatibility,
``minispeed/flat.py:50-89``): the group's parameters are concatenated in
order into ``numel`` elements, padded at the end to ``numel_padded``, a
multiple of the world size; rank ``r`` owns ``[r*shard_size,
(r+1)*shard_size)`` (stage 0: every rank owns the whole buffer).

What differs from the reference is where the model-dtype tensors live.  The
reference keeps each ``p.data`` and ``p.grad`` as a separate tensor and
copies them into and out of the fp32 buffers with one copy per parameter
(``flat.py:115-213``).  Here every ``p.data`` is a *view* into one
model-dtype arena (``param_arena``) and every ``p.grad`` a view into one
model-dtype gradient arena (``grad_arena``) with the same flat layout as the
fp32 masters.  Consequences on the GPU:

* autograd accumulates gradients straight into the arena, so "flatten" is
  free and the fused kernels read one flat buffer (peers read it over NVLink);
* the AdamW kernel writes the cast parameters straight into ``param_arena``
  (or into the peers' arenas), so "copy flat to model" is free;
* the flat range arithmetic below works on arena slices instead of
  per-parameter copies.

Buffers:
  ``data``        fp32 masters, full (stages 0-2) or this rank's shard
                  (stage 3 after :meth:`partition_params`);
  ``param_arena`` model-dtype full buffer backing the params (stage 3: only
                  while gathered);
  ``param_shard`` stage 3: shard-sized model-dtype buffer backing the flat
                  placeholders while the params are freed;
  ``grad_arena``  model-dtype full buffer backing ``p.grad``;
  ``grad``        fp32 full reduction buffer (library path and stage 0 only);
  ``grad_shard``  fp32 reduced gradient shard (stages 2-3).
"""

from __future__ import annotations

from typing import Iterable, List, Optional, Sequence, Tuple

import torch
from torch import nn


def _round_up(x: int, multiple: int) -> int:
    return -(-x // multiple) * multiple


class FlatParamGroup:
    def __init__(self, params: Sequence[nn.Parameter], *, rank: int, world_size: int,
                 zero_stage: int, device: torch.device):
        params = list(params)
        if not params:
            raise ValueError("FlatParamGroup requires at least one parameter")
        self.params: List[nn.Parameter] = params
        self.rank = int(rank)
        self.world_size = int(world_size)
        self.zero_stage = int(zero_stage)
        self.device = torch.device(device)

        self._numels = [p.numel() for p in params]
        self._shapes = [tuple(p.shape) for p in params]
        self._offsets_int: List[int] = []
        off = 0
        for n in self._numels:
            self._offsets_int.append(off)
            off += n
        # reference-compatible (offset, param) table
        self._offsets: List[Tuple[int, nn.Parameter]] = list(zip(self._offsets_int, params))
        self.numel = off
        self.numel_padded = _round_up(self.numel, self.world_size)
        self.shard_size = self.numel_padded // self.world_size
        if self.zero_stage >= 1:
            self.shard_start = self.rank * self.shard_size
            self.shard_end = self.shard_start + self.shard_size
        else:
            self.shard_start, self.shard_end = 0, self.numel_padded

        self.data = torch.zeros(self.numel_padded, dtype=torch.float32, device=self.device)
        # fp32 reduction buffers are allocated on first use: the fused GPU
        # path at world size 1 never needs them
        self._grad: Optional[torch.Tensor] = None
        self._grad_shard: Optional[torch.Tensor] = None

        self.param_dtype: torch.dtype = params[0].dtype
        self.param_arena: Optional[torch.Tensor] = None
        self.param_shard: Optional[torch.Tensor] = None
        self.grad_arena: Optional[torch.Tensor] = None
        self._grad_views: Optional[List[torch.Tensor]] = None   # tensors bind_grads put in p.grad
        self._grad_views_of: Optional[torch.Tensor] = None      # ... as views of this arena
        # a pinned gradient arena (peer heap) is zeroed between windows,
        # never freed, so peers can keep addressing it
        self._arena_pinned = False
        self._partitioned = False
        self._bind_full(self._new_arena_from_params(self.param_dtype))

    # ----------------------------------------------------------- arena views
    def _new_arena_from_params(self, dtype: torch.dtype) -> torch.Tensor:
        arena = torch.zeros(self.numel_padded, dtype=dtype, device=self.device)
        with torch.no_grad():
            for off, n, p in zip(self._offsets_int, self._numels, self.params):
                arena[off:off + n].copy_(p.data.reshape(-1))
        return arena

    def _bind_full(self, arena: torch.Tensor) -> None:
        """Point every ``p.data`` at its full-shaped view of ``arena``."""
        self.param_arena = arena
        for off, n, shape, p in zip(self._offsets_int, self._numels, self._shapes, self.params):
            p.data = arena[off:off + n].view(shape)

    def _placeholder_range(self, i: int) -> Tuple[int, int]:
        off, n = self._offsets_int[i], self._numels[i]
        lo = max(off, self.shard_start)
        hi = min(off + n, self.shard_end)
        return lo, max(lo, hi)

    def _bind_placeholders(self) -> None:
        """Point every ``p.data`` at its locally owned slice of ``param_shard``."""
        s0 = self.shard_start
        for i, p in enumerate(self.params):
            lo, hi = self._placeholder_range(i)
            p.data = self.param_shard[lo - s0:hi - s0]

    def bound(self) -> bool:
        """True when every param still aliases this group's arena.

        A user may rebind ``p.data`` (``module.to(...)``); the engine checks
        this once per step and rebinds by copying.
        """
        if self._partitioned and self.param_arena is None:
            return True
        base = self.param_arena.data_ptr()
        esz = self.param_arena.element_size()
        dt = self.param_dtype
        # Parameter.data_ptr() directly: no .data alias object per check
        for off, p in zip(self._offsets_int, self.params):
            if p.data_ptr() != base + off * esz or p.dtype != dt:
                return False
        return True

    def grads_bound(self) -> bool:
        """True when every ``p.grad`` is still the arena view
        :meth:`bind_grads` assigned (an identity check, no tensor calls)."""
        views = self._grad_views
        if views is None or self._grad_views_of is not self.grad_arena:
            return False
        for p, v in zip(self.params, views):
            if p.grad is not v:
                return False
        return True

    def rebind(self) -> None:
        if not self.bound():
            self._bind_full(self._new_arena_from_params(self.param_dtype))

    def cast_params(self, dtype: torch.dtype) -> None:
        """Re-home the params in an arena of the training dtype (values cast)."""
        if dtype == self.param_dtype and self.param_arena is not None:
            return
        arena = self.param_arena.to(dtype)
        self.param_dtype = dtype
        self._bind_full(arena)
        self.grad_arena = None

    # ------------------------------------------------------------ ranges
    @property
    def master_range(self) -> Tuple[int, int]:
        """Flat range covered by ``data``."""
        if self._partitioned:
            return self.shard_start, self.shard_end
        return 0, self.numel_padded

    def _model_view(self) -> Tuple[torch.Tensor, int]:
        """(buffer holding the current model params, flat index of its element 0)."""
        if self._partitioned and self.param_arena is None:
            return self.param_shard, self.shard_start
        return self.param_arena, 0

    @torch.no_grad()
    def copy_model_to_flat(self) -> None:
        """Snapshot the model params covered by ``data`` into the fp32 masters."""
        buf, base = self._model_view()
        ms, me = self.master_range
        lo, hi = max(ms, base), min(me, base + buf.numel())
        if lo < hi:
            self.data[lo - ms:hi - ms].copy_(buf[lo - base:hi - base])

    @torch.no_grad()
    def copy_flat_to_model(self, full_flat: Optional[torch.Tensor] = None) -> None:
        """Write masters (or a full ``[0, numel_padded)`` buffer) into the params."""
        if full_flat is not None:
            src, sbase = full_flat, 0
        else:
            src, sbase = self.data, self.master_range[0]
        dst, dbase = self._model_view()
        lo = max(sbase, dbase)
        hi = min(sbase + src.numel(), dbase + dst.numel())
        if lo < hi:
            dst[lo - dbase:hi - dbase].copy_(src[lo - sbase:hi - sbase])

    # ------------------------------------------------------- stage-3 params
    @torch.no_grad()
    def partition_params(self) -> None:
        """Keep only this rank's fp32 shard; params become flat placeholders."""
        if self._partitioned:
            return
        self.data = self.data[self.shard_start:self.shard_end].clone()
        self._partitioned = True
        self.param_shard = torch.zeros(self.shard_size, dtype=self.param_dtype,
                                       device=self.device)
        self.dematerialize_params()
        self.copy_flat_to_model()

    @torch.no_grad()
    def materialize_params(self) -> None:
        """Give every param an (uninitialised) full-shaped tensor to fill."""
        if not self._partitioned:
            return
        if self.param_arena is None:
            self._bind_full(torch.empty(self.numel_padded, dtype=self.param_dtype,
                                        device=self.device))
        if self.grad_arena is not None:
            self.bind_grads()

    @torch.no_grad()
    def dematerialize_params(self) -> None:
        """Drop the full params back to their locally owned flat slices."""
        if not self._partitioned:
            return
        for p in self.params:
            p.grad = None
        self.param_arena = None
        self._bind_placeholders()

    @property
    def params_materialized(self) -> bool:
        return self.param_arena is not None

    # ----------------------------------------------------------------- grads
    @property
    def grad(self) -> Optional[torch.Tensor]:
        """fp32 full gradient buffer (stages 0-2 always present; stage 3 only
        between flatten and reduce-scatter)."""
        if self._grad is None and self.zero_stage < 3:
            self._grad = torch.zeros(self.numel_padded, dtype=torch.float32, device=self.device)
        return self._grad

    @grad.setter
    def grad(self, value: Optional[torch.Tensor]) -> None:
        self._grad = value

    @property
    def grad_shard(self) -> Optional[torch.Tensor]:
        """fp32 reduced gradient shard (stages 2-3)."""
        if self.zero_stage < 2:
            return None
        if self._grad_shard is None:
            self._grad_shard = torch.zeros(self.shard_size, dtype=torch.float32,
                                           device=self.device)
        return self._grad_shard

    def ensure_grad_arena(self) -> torch.Tensor:
        """Allocate (zeroed) and bind the model-dtype gradient arena."""
        if self.grad_arena is None:
            self.grad_arena = torch.zeros(self.numel_padded, dtype=self.param_dtype,
                                          device=self.device)
            self._grad_views = None
        if self.param_arena is not None and not self.grads_bound():
            self.bind_grads()
        return self.grad_arena

    def bind_grads(self) -> None:
        ga = self.grad_arena
        views = []
        for off, n, shape, p in zip(self._offsets_int, self._numels, self._shapes, self.params):
            v = ga[off:off + n].view(shape)
            p.grad = v
            views.append(p.grad)
        self._grad_views = views
        self._grad_views_of = ga

    @torch.no_grad()
    def collect_grads(self) -> torch.Tensor:
        """Make ``grad_arena`` hold every param's accumulated gradient.

        Gradients that autograd wrote somewhere else (the user reset
        ``p.grad``, or it was never bound) are copied in; params without a
        gradient contribute zeros.  Returns the arena.
        """
        ga = self.grad_arena
        if ga is None:
            ga = self.grad_arena = torch.zeros(self.numel_padded, dtype=self.param_dtype,
                                               device=self.device)
            self._grad_views = None
            fresh = True
        else:
            if self.grads_bound():
                return ga       # every gradient already accumulated in place
            fresh = False
        base = ga.data_ptr()
        esz = ga.element_size()
        for off, n, p in zip(self._offsets_int, self._numels, self.params):
            g = p.grad
            if g is None:
                if not fresh:
                    ga[off:off + n].zero_()
                continue
            if g.data_ptr() == base + off * esz and g.dtype == ga.dtype:
                continue
            ga[off:off + n].copy_(g.reshape(-1))
        return ga

    @torch.no_grad()
    def flatten_grads(self) -> None:
        """Library path: the fp32 ``grad`` buffer receives the gradients.

        Matches the reference contract (``flat.py:196-213``): afterwards
        ``grad`` holds every param gradient in fp32 (zeros where absent).
        """
        ga = self.collect_grads()
        if self.grad is None:
            self.grad = torch.empty(self.numel_padded, dtype=torch.float32, device=self.device)
        self.grad.copy_(ga)

    @torch.no_grad()
    def zero_grad(self) -> None:
        """Start a new accumulation window."""
        if self._grad is not None:
            if self.zero_stage >= 3:
                self._grad = None
            else:
                self._grad.zero_()
        if self._grad_shard is not None:
            self._grad_shard.zero_()
        if self.grad_arena is not None:
            if self.zero_stage >= 3 and not self._arena_pinned:
                self.grad_arena = None
                for p in self.params:
                    p.grad = None
            else:
                self.grad_arena.zero_()
                if self.param_arena is not None and not self.grads_bound():
                    self.bind_grads()

    def grad_for_shard(self) -> torch.Tensor:
        if self.grad_shard is not None:
            return self.grad_shard
        return self.grad[self.shard_start:self.shard_end]

    def local_grad_sumsq(self) -> torch.Tensor:
        g = self.grad_for_shard()
        return g.float().pow(2).sum()

    @property
    def shard(self) -> torch.Tensor:
        if self._partitioned:
            return self.data
        return self.data[self.shard_start:self.shard_end]

    @torch.no_grad()
    def unscale_grads(self, scale: float) -> None:
        if scale != 1.0 and self.grad is not None:
            self.grad.div_(scale)

    @torch.no_grad()
    def scale_grads(self, factor: float) -> None:
        if factor == 1.0:
            return
        if self.grad_shard is not None:
            self.grad_shard.mul_(factor)
        elif self.grad is not None:
            self.grad.mul_(factor)

    def numel_shard(self) -> int:
        return self.shard_end - self.shard_start

    def param_index_ranges(self) -> List[Tuple[int, int]]:
        """Flat ``[start, end)`` of each parameter, in group order."""
        return [(o, o + n) for o, n in zip(self._offsets_int, self._numels)]


def build_flat_groups(param_groups: Iterable[dict], *, rank: int, world_size: int,
                      zero_stage: int, device: torch.device
                      ) -> Tuple[List[FlatParamGroup], List[dict]]:
    """torch-style group dicts -> (flat groups, per-group option dicts)."""
    flat, options = [], []
    for group in param_groups:
        params = [p for p in group["params"] if p.requires_grad]
        if not params:
            continue
        flat.append(FlatParamGroup(params, rank=rank, world_size=world_size,
                                   zero_stage=zero_stage, device=device))
        options.append({k: v for k, v in group.items() if k != "params"})
    if not flat:
        raise ValueError("No trainable parameters found")
    return flat, options
