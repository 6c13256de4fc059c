"""Python API of the step-pipeline kernels.

CUDA tensors run the sm_100a kernels of ``minispeed_b200._C``; CPU tensors
run the PyTorch statements that define what each kernel computes (they are
also the fp32 oracle of the GPU numerics tests).

Reference: AdamW on the flat fp32 shard (``minispeed/optim/adam.py:60-93``),
the overflow check and its all-reduce (``minispeed/precision.py:79-92``),
gradient flattening, unscaling and the shard's sum of squares
(``minispeed/flat.py:197-257``), and the fp32 -> model-dtype copy back into the
parameters (``minispeed/flat.py:134-156``).  Here each of those is one fused
kernel over the flat arenas.
"""

from __future__ import annotations

from typing import Iterable, List, Optional, Tuple

import torch

from . import _ext

STATS_SLOTS = 1 << 16  # per-block partials of one optimizer step
OUT_FLAG, OUT_SUMSQ, OUT_NORM, OUT_COEF = 0, 1, 2, 3


class StepStats:
    """Device accumulator of one step's gradient statistics.

    :meth:`accumulate` runs the fused stats kernel over a gradient buffer,
    writing one (sum-of-squares, inf/nan flag) partial per thread block into
    a scratch array; :meth:`finalize` folds all partials of the step in a fixed
    order into ``out = [flag, sumsq, norm, clip_coef]`` (bitwise reproducible).
    Nothing here synchronizes with the host.
    """

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.out = torch.zeros(8, dtype=torch.float32, device=self.device)
        if self.device.type == "cuda":
            self.partials = torch.zeros(STATS_SLOTS, dtype=torch.float32, device=self.device)
            self.flags = torch.zeros(STATS_SLOTS, dtype=torch.int32, device=self.device)
        self.used = 0
        self._cpu_sumsq = 0.0
        self._cpu_bad = False

    def reset(self) -> None:
        self.used = 0
        self._cpu_sumsq = 0.0
        self._cpu_bad = False

    def accumulate(self, x: torch.Tensor, mul: float = 1.0) -> None:
        if x.numel() == 0:
            return
        if x.is_cuda:
            left = STATS_SLOTS - self.used
            if left < 1:
                raise RuntimeError("StepStats scratch exhausted; too many buffers in one step")
            self.used += int(_ext.get().grad_stats(x, float(mul), self.partials, self.flags,
                                                   self.used, min(left, 148 * 8)))
        else:
            f = x.detach().float()
            self._cpu_bad |= not bool(torch.isfinite(f).all())
            self._cpu_sumsq += float((f * mul).pow(2).sum())

    def finalize(self, max_norm: Optional[float], epilogue: bool = True) -> torch.Tensor:
        mn = float(max_norm) if max_norm else 0.0
        if self.device.type == "cuda":
            if self.used == 0:
                self.out.zero_()
                if epilogue:
                    _ext.get().stats_epilogue(self.out, mn)
            else:
                _ext.get().stats_finalize(self.partials, self.flags, self.used, self.out, mn,
                                          epilogue)
        else:
            self.out[OUT_FLAG] = 1.0 if self._cpu_bad else 0.0
            self.out[OUT_SUMSQ] = self._cpu_sumsq
            if epilogue:
                epilogue_cpu(self.out, mn)
        return self.out

    def epilogue(self, max_norm: Optional[float]) -> torch.Tensor:
        mn = float(max_norm) if max_norm else 0.0
        if self.out.is_cuda:
            _ext.get().stats_epilogue(self.out, mn)
        else:
            epilogue_cpu(self.out, mn)
        return self.out


def epilogue_cpu(out: torch.Tensor, max_norm: float) -> None:
    out[OUT_FLAG] = 1.0 if float(out[OUT_FLAG]) > 0 else 0.0
    norm = float(torch.sqrt(out[OUT_SUMSQ]))
    out[OUT_NORM] = norm
    coef = 1.0
    if max_norm > 0 and norm > max_norm:
        coef = max_norm / (norm + 1e-6)
    out[OUT_COEF] = coef


def grad_stats(tensors: Iterable[torch.Tensor], inv_scale: float = 1.0
               ) -> Tuple[torch.Tensor, torch.Tensor]:
    """(flag, sum of squares of ``t*inv_scale``) over all tensors, on device."""
    tensors = [t for t in tensors if t is not None]
    dev = tensors[0].device if tensors else torch.device("cpu")
    st = StepStats(dev)
    for t in tensors:
        st.accumulate(t.contiguous(), inv_scale)
    out = st.finalize(None)
    return out[OUT_FLAG], out[OUT_SUMSQ]


def adamw_step(master: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor,
               grad: torch.Tensor, *, lr: float, beta1: float, beta2: float, eps: float,
               wd: float, bc1: float, bc2: float, grad_mul: float = 1.0,
               stats: Optional[torch.Tensor] = None, max_norm: Optional[float] = None,
               param_out: Optional[torch.Tensor] = None, peer=None) -> None:
    """One fused AdamW update of an fp32 shard (see ``optim/adam.py``).

    ``stats`` (finalized :class:`StepStats` output) makes the kernel skip the
    update when the step overflowed and scale the gradient by the clip
    coefficient; ``param_out`` receives the model-dtype cast of the updated
    master.  ``peer`` is reserved for the fused all-gather variant.
    """
    if peer is not None:
        raise NotImplementedError("peer all-gather variant is provided by parallel.fused")
    if master.is_cuda:
        _ext.get().adamw(master, exp_avg, exp_avg_sq, grad, param_out, stats, float(lr),
                         float(beta1), float(beta2), float(eps), float(wd), float(bc1),
                         float(bc2), float(grad_mul))
        return
    adamw_reference(master, exp_avg, exp_avg_sq, grad, lr=lr, beta1=beta1, beta2=beta2,
                    eps=eps, wd=wd, bc1=bc1, bc2=bc2, grad_mul=grad_mul, stats=stats,
                    param_out=param_out)


@torch.no_grad()
def adamw_reference(master, exp_avg, exp_avg_sq, grad, *, lr, beta1, beta2, eps, wd, bc1, bc2,
                    grad_mul=1.0, stats=None, param_out=None) -> None:
    """fp32 PyTorch definition of the fused AdamW kernel."""
    coef = 1.0
    if stats is not None:
        if float(stats[OUT_FLAG]) != 0.0:
            return
        coef = float(stats[OUT_COEF])
    g = grad.float() * grad_mul
    if coef != 1.0:
        g = g * coef
    if wd != 0.0:
        master.add_(master, alpha=-lr * wd)
    exp_avg.mul_(beta1).add_(g, alpha=1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    denom = (exp_avg_sq / bc2).sqrt().add_(eps)
    master.addcdiv_(exp_avg / bc1, denom, value=-lr)
    if param_out is not None:
        param_out.copy_(master)


def cast_scale(src: torch.Tensor, dst: torch.Tensor, mul: float = 1.0) -> torch.Tensor:
    """``dst = dtype(dst)(float(src) * mul)``."""
    if src.is_cuda:
        _ext.get().cast_scale(src, dst, float(mul))
    else:
        dst.copy_(src.float() * mul if mul != 1.0 else src)
    return dst


def flat_views(buf: torch.Tensor, sizes: List[int]) -> List[torch.Tensor]:
    out, off = [], 0
    for n in sizes:
        out.append(buf[off:off + n])
        off += n
    return out
