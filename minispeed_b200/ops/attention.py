"""Causal self-attention (forward + backward) on [B, T, H, D] tensors.

The sm_100a flash-attention kernel (``csrc/attention.cu``) is used when the
extension provides it: blockwise online softmax, causal tile skipping, GQA
by head mapping, q/k/v read straight from the fused qkv projection layout
and the output written in the [B, T, H*D] layout the output projection
consumes.  ``MSB_ATTN=torch`` selects PyTorch's SDPA instead (comparison
baseline in the tests).
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from . import _ext

_MODE = os.environ.get("MSB_ATTN", "auto")


def _sdpa(q, k, v):
    H, Hkv = q.shape[2], k.shape[2]
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
    if Hkv != H:
        rep = H // Hkv
        kt = kt.repeat_interleave(rep, dim=1)
        vt = vt.repeat_interleave(rep, dim=1)
    o = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True)
    return o.transpose(1, 2)


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    if q.is_cuda and _MODE != "torch" and hasattr(_ext.get(), "attn_fwd"):
        from .flash import flash_attention

        return flash_attention(q, k, v)
    return _sdpa(q, k, v)
