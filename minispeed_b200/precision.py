"""Mixed precision: the dynamic loss-scale state machine and overflow checks.

State machine (reference ``minispeed/precision.py:10-76``): the scale starts
at ``2**initial_scale_power`` (or at a positive ``loss_scale``), doubles after
``scale_window`` consecutive clean steps (capped at ``2**24``) and halves on
an inf/nan step (floored at 1) which is then skipped.  A positive static
``loss_scale`` still adapts, as in the reference.  Disabled (fp32/bf16) means
a constant factor of 1.

On the GPU the overflow test itself is not done here: it is one output of
the fused gradient-statistics kernel (``ops.grad_stats``), which produces the
inf/nan flag and the sum of squares in one pass over the gradients, leaving
them in device memory for the AdamW kernel to consume without a host round
trip.  :func:`has_overflow` is the standalone host-facing check.
"""

from __future__ import annotations

import torch

from . import comm


class DynamicLossScaler:
    def __init__(self, enabled: bool = True, init_scale: float = 0.0,
                 scale_window: int = 1000, min_scale: float = 1.0,
                 max_scale: float = 2.0 ** 24):
        self.enabled = bool(enabled)
        self.min_scale = float(min_scale)
        self.max_scale = float(max_scale)
        self.scale_window = max(1, int(scale_window))
        if self.enabled and init_scale and init_scale > 0:
            self.scale = float(init_scale)
        else:
            self.scale = 1.0
        self.good_steps = 0
        self.skipped_steps = 0

    def set_scale_from_power(self, power: int) -> None:
        if self.enabled:
            self.scale = float(2.0 ** int(power))

    @property
    def loss_scale_factor(self) -> float:
        return self.scale if self.enabled else 1.0

    def update(self, overflow: bool) -> None:
        """Advance the scaler after a step: halve on overflow (and count the skip),
        double after ``scale_window`` consecutive good steps."""
        if not self.enabled:
            return
        if overflow:
            self.scale = max(self.scale * 0.5, self.min_scale)
            self.good_steps = 0
            self.skipped_steps += 1
            return
        self.good_steps += 1
        if self.good_steps >= self.scale_window and self.scale < self.max_scale:
            self.scale = min(self.scale * 2.0, self.max_scale)
            self.good_steps = 0

    def state_dict(self) -> dict:
        return {"enabled": self.enabled, "scale": self.scale,
                "good_steps": self.good_steps, "skipped_steps": self.skipped_steps}

    def load_state_dict(self, state: dict) -> None:
        self.enabled = bool(state.get("enabled", self.enabled))
        self.scale = float(state.get("scale", self.scale))
        self.good_steps = int(state.get("good_steps", 0))
        self.skipped_steps = int(state.get("skipped_steps", 0))


def has_overflow(*buffers: torch.Tensor) -> bool:
    """True when any element of any given tensor is inf or nan."""
    for buf in buffers:
        if buf is None or buf.numel() == 0:
            continue
        if buf.is_cuda:
            from .ops import kernels

            flag, _ = kernels.grad_stats([buf], inv_scale=1.0)
            if bool(flag.item()):
                return True
        elif not bool(torch.isfinite(buf).all()):
            return True
    return False


def global_overflow(local_overflow: bool) -> bool:
    """OR a local overflow flag over every data-parallel rank."""
    return comm.all_reduce_flag(local_overflow)
