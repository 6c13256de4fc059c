"""AdamW over the flat fp32 master shard of each parameter group.

Math and operation order follow the reference (``minispeed/optim/adam.py:59-93``)
so that fp32 masters stay bitwise-close to it:

    p  <- p + (-lr*wd) * p                 (decoupled weight decay, first)
    m  <- b1*m + (1-b1)*g
    v  <- b2*v + (1-b2)*g*g
    p  <- p + (-lr) * (m/bc1) / (sqrt(v/bc2) + eps)

with ``bc_i = 1 - b_i**step``.  "Adam" in the config runs the same decoupled
update.  The moments cover only this rank's ZeRO shard.

On the GPU the whole update is ONE kernel per group
(:func:`minispeed_b200.ops.kernels.adamw_step`) that also

* reads the gradient in whatever dtype it lives in (model-dtype arena at
  world size 1, fp32 reduced shard otherwise) and applies the unscale and
  clip factors on the fly (the clip coefficient is computed on the device
  from the fused gradient statistics, so no host round trip sits between
  the norm and the update),
* skips the update on the device when the step's inf/nan flag is set, and
* writes the fp32->fp16/bf16 cast of the new masters straight into the
  parameter arena (or, with the fused collectives, into every peer's).

The PyTorch path below (CPU, and the library-collective path) keeps the
reference's sequence of tensor ops.
"""

from __future__ import annotations

from typing import List, Optional

import torch

from ..flat import FlatParamGroup


class FlatAdam:
    def __init__(self, flat_groups: List[FlatParamGroup], option_groups: List[dict],
                 zero_stage: int = 0):
        self.flat_groups = flat_groups
        self.zero_stage = zero_stage
        self.param_groups: List[dict] = []
        self._state: List[dict] = []
        for flat, opts in zip(flat_groups, option_groups):
            group = dict(opts)
            group.setdefault("lr", 1e-3)
            group.setdefault("betas", (0.9, 0.999))
            group.setdefault("eps", 1e-8)
            group.setdefault("weight_decay", 0.0)
            self.param_groups.append(group)
            n = flat.numel_shard()
            dev = flat.data.device
            self._state.append({
                "step": 0,
                "exp_avg": torch.zeros(n, dtype=torch.float32, device=dev),
                "exp_avg_sq": torch.zeros(n, dtype=torch.float32, device=dev),
            })

    @property
    def state(self) -> List[dict]:
        return self._state

    @staticmethod
    def hyper(group: dict, step: int):
        lr = float(group["lr"])
        b1, b2 = (float(b) for b in group["betas"])
        eps = float(group["eps"])
        wd = float(group.get("weight_decay", 0.0))
        return lr, b1, b2, eps, wd, 1.0 - b1 ** step, 1.0 - b2 ** step

    # ------------------------------------------------------ library path
    @torch.no_grad()
    def step(self) -> bool:
        """Update each group's shard from ``grad_for_shard()`` (already reduced,
        unscaled and clipped).  Used on CPU and by the library-collective path."""
        for group, flat, st in zip(self.param_groups, self.flat_groups, self._state):
            shard = flat.shard
            grad = flat.grad_for_shard()
            if grad.shape != shard.shape:
                raise RuntimeError(f"grad/shard shape mismatch: {grad.shape} vs {shard.shape}")
            st["step"] += 1
            lr, b1, b2, eps, wd, bc1, bc2 = self.hyper(group, st["step"])
            if shard.is_cuda:
                from ..ops import kernels

                kernels.adamw_step(shard, st["exp_avg"], st["exp_avg_sq"], grad,
                                   lr=lr, beta1=b1, beta2=b2, eps=eps, wd=wd,
                                   bc1=bc1, bc2=bc2)
                continue
            m, v = st["exp_avg"], st["exp_avg_sq"]
            if wd != 0.0:
                shard.add_(shard, alpha=-lr * wd)
            m.mul_(b1).add_(grad, alpha=1.0 - b1)
            v.mul_(b2).addcmul_(grad, grad, value=1.0 - b2)
            denom = (v / bc2).sqrt().add_(eps)
            shard.addcdiv_(m / bc1, denom, value=-lr)
        return True

    # ------------------------------------------------------- fused path
    @torch.no_grad()
    def fused_step(self, grads: List[torch.Tensor], stats: torch.Tensor,
                   grad_mul: float, max_norm: Optional[float],
                   param_outs: List[Optional[torch.Tensor]], fanouts=None) -> None:
        """Enqueue the device-skipping fused update for every group.

        ``grads[i]`` is group i's gradient covering its shard (any float
        dtype), scaled by ``grad_mul`` inside the kernel; ``stats`` is the
        finalized device statistics tensor (flag, sum of squares, norm,
        clip coefficient).  ``fanouts[i]``, when given, makes the kernel
        store the cast parameters into every rank's parameter arena over
        NVLink (the fused all-gather).  The step counters advance on the host
        only once the caller knows the step was applied (:meth:`commit_step`).
        """
        from ..ops import _ext, kernels

        for i, (group, flat, st) in enumerate(zip(self.param_groups, self.flat_groups,
                                                   self._state)):
            lr, b1, b2, eps, wd, bc1, bc2 = self.hyper(group, st["step"] + 1)
            fan = None if fanouts is None else fanouts[i]
            if fan is not None:
                heaps, param_off, pdtype, s0, world = fan
                _ext.get().adamw_fanout(flat.shard, st["exp_avg"], st["exp_avg_sq"], grads[i],
                                        heaps, param_off, pdtype, s0, world, stats, lr, b1, b2,
                                        eps, wd, bc1, bc2, grad_mul)
                continue
            kernels.adamw_step(flat.shard, st["exp_avg"], st["exp_avg_sq"], grads[i],
                               lr=lr, beta1=b1, beta2=b2, eps=eps, wd=wd, bc1=bc1, bc2=bc2,
                               grad_mul=grad_mul, stats=stats,
                               max_norm=max_norm, param_out=param_outs[i])

    def commit_step(self) -> None:
        for st in self._state:
            st["step"] += 1

    # -------------------------------------------------------------- state
    def zero_grad(self) -> None:
        for flat in self.flat_groups:
            flat.zero_grad()

    def state_dict(self) -> dict:
        return {
            "param_groups": [dict(g) for g in self.param_groups],
            "shard_state": [{"step": st["step"], "exp_avg": st["exp_avg"].clone(),
                             "exp_avg_sq": st["exp_avg_sq"].clone()} for st in self._state],
        }

    def load_state_dict(self, state_dict: dict) -> None:
        for saved, group in zip(state_dict["param_groups"], self.param_groups):
            group.update({k: v for k, v in saved.items() if k != "params"})
        for saved, st in zip(state_dict["shard_state"], self._state):
            st["step"] = int(saved["step"])
            st["exp_avg"].copy_(saved["exp_avg"])
            st["exp_avg_sq"].copy_(saved["exp_avg_sq"])
