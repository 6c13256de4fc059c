"""Activation checkpointing (recompute in backward).

Same API as the reference helper (``minispeed/activation_checkpointing.py:17-30``):
``checkpoint(fn, *args)`` and ``checkpoint_sequential(functions, segments,
input)``, non-reentrant by default.  The model blocks of
:mod:`minispeed_b200.models` call :func:`checkpoint` per block when built
with ``activation_checkpointing=True``; their fused kernels are simply run
again in the recompute.
"""

from __future__ import annotations

import torch
from torch.utils.checkpoint import checkpoint as _checkpoint
from torch.utils.checkpoint import checkpoint_sequential as _checkpoint_sequential


def checkpoint(function, *args, **kwargs):
    use_reentrant = kwargs.pop("use_reentrant", False)
    return _checkpoint(function, *args, use_reentrant=use_reentrant, **kwargs)


def checkpoint_sequential(functions, *args, **kwargs):
    use_reentrant = kwargs.pop("use_reentrant", False)
    return _checkpoint_sequential(functions, *args, use_reentrant=use_reentrant, **kwargs)


__all__ = ["checkpoint", "checkpoint_sequential"]

# keep torch importable name for type checkers
_ = torch
