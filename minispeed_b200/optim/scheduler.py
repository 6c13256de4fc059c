"""Learning-rate schedules in the DeepSpeed config schema.

The engine steps a schedule once per applied (non-skipped) optimizer step,
after the update, so the first update runs with the optimizer's configured
``lr`` (reference ``minispeed/optim/scheduler.py:31,50-54`` and
``engine.py:319``).  A schedule writes one lr into every parameter group.

* ``WarmupLR`` (alias ``WarmupLRConst``/``ConstantLR``): linear from
  ``warmup_min_lr`` to ``warmup_max_lr`` over ``warmup_num_steps`` steps,
  then constant.
* ``WarmupDecayLR``: the same warmup, then linear decay that reaches
  ``warmup_min_lr`` at ``total_num_steps`` and stays there.

``state_dict`` stores the schedule type and parameters; loading restores the
step counter only (``scheduler.py:59-70``).
"""

from __future__ import annotations

from typing import Optional


class _Schedule:
    def __init__(self, optimizer, warmup_min_lr: float = 0.0,
                 warmup_max_lr: float = 1e-3, warmup_num_steps: int = 0,
                 total_num_steps: Optional[int] = None):
        self.optimizer = optimizer
        self.warmup_min_lr = float(warmup_min_lr)
        self.warmup_max_lr = float(warmup_max_lr)
        self.warmup_num_steps = max(0, int(warmup_num_steps))
        self.total_num_steps = None if total_num_steps is None else int(total_num_steps)
        self.last_epoch = -1
        self.base_lrs = [float(g.get("lr", self.warmup_max_lr)) for g in optimizer.param_groups]

    def _ramp(self, epoch: int) -> float:
        n = self.warmup_num_steps
        if n <= 0 or epoch >= n:
            return self.warmup_max_lr
        return self.warmup_min_lr + (self.warmup_max_lr - self.warmup_min_lr) * (epoch / n)

    def get_lr(self) -> float:  # pragma: no cover - abstract
        raise NotImplementedError

    def step(self, epoch: Optional[int] = None) -> None:
        self.last_epoch = self.last_epoch + 1 if epoch is None else int(epoch)
        lr = self.get_lr()
        for group in self.optimizer.param_groups:
            group["lr"] = lr

    def get_last_lr(self) -> float:
        return float(self.optimizer.param_groups[0]["lr"])

    def state_dict(self) -> dict:
        return {"type": type(self).__name__, "last_epoch": self.last_epoch,
                "warmup_min_lr": self.warmup_min_lr, "warmup_max_lr": self.warmup_max_lr,
                "warmup_num_steps": self.warmup_num_steps,
                "total_num_steps": self.total_num_steps}

    def load_state_dict(self, state: dict) -> None:
        self.last_epoch = int(state["last_epoch"])


class WarmupLR(_Schedule):
    def get_lr(self) -> float:
        return self._ramp(self.last_epoch)


class WarmupDecayLR(_Schedule):
    def get_lr(self) -> float:
        e = self.last_epoch
        if e < self.warmup_num_steps:
            return self._ramp(e)
        total = self.total_num_steps
        if total is None:
            return self.warmup_max_lr
        if e >= total:
            return self.warmup_min_lr
        remaining = (total - e) / max(1, total - self.warmup_num_steps)
        return self.warmup_min_lr + (self.warmup_max_lr - self.warmup_min_lr) * remaining


class ConstantLR(WarmupLR):
    """Config alias of :class:`WarmupLR`."""


def build_scheduler(optimizer, scheduler_type: str, params: dict):
    """The scheduler named by the config (``WarmupLR`` and its aliases, or
    ``WarmupDecayLR``) over ``optimizer.param_groups``."""
    kwargs = dict(warmup_min_lr=params.get("warmup_min_lr", 0.0),
                  warmup_max_lr=params.get("warmup_max_lr"),
                  warmup_num_steps=params.get("warmup_num_steps", 0),
                  total_num_steps=params.get("total_num_steps"))
    if kwargs["warmup_max_lr"] is None:
        kwargs["warmup_max_lr"] = float(optimizer.param_groups[0].get("lr", 1e-3))
    if scheduler_type in ("WarmupLR", "WarmupLRConst", "ConstantLR"):
        return WarmupLR(optimizer, **kwargs)
    if scheduler_type == "WarmupDecayLR":
        return WarmupDecayLR(optimizer, **kwargs)
    raise ValueError(f"Unknown scheduler type: {scheduler_type}")
