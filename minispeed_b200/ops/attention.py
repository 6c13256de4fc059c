"""Causal self-attention (forward + backward) over a fused qkv projection.

``attention_qkv(qkv)`` takes the [B, T, 3, H, D] output of the fused qkv
projection and returns [B, T, H*D], the layout the output projection
consumes.  Its backward writes dq, dk and dv into ONE [B, T, 3, H, D]
buffer with a single kernel; going through three views of the qkv tensor
instead would make autograd materialize three zero-filled full-size
gradients and add them (3 fills + 3 copies + 2 adds per layer).

The attention core is PyTorch's scaled_dot_product_attention (the cuDNN
sm_100 flash kernels), run on strided [B, H, T, D] views without copies.
GQA (fewer kv heads) is handled by :func:`causal_attention`.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _sdpa(q, k, v):
    H, Hkv = q.shape[2], k.shape[2]
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
    if Hkv != H:
        rep = H // Hkv
        kt = kt.repeat_interleave(rep, dim=1)
        vt = vt.repeat_interleave(rep, dim=1)
    o = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True)
    return o.transpose(1, 2)


class _AttnQKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv):
        B, T, _, H, D = qkv.shape
        with torch.enable_grad():
            leaves = [qkv[:, :, i].detach().transpose(1, 2).requires_grad_() for i in range(3)]
            o = F.scaled_dot_product_attention(*leaves, is_causal=True)
        ctx.graph = (leaves, o)
        ctx.shape = (B, T, H, D)
        return o.detach().transpose(1, 2).reshape(B, T, H * D)

    @staticmethod
    def backward(ctx, dout):
        leaves, o = ctx.graph
        B, T, H, D = ctx.shape
        g = dout.reshape(B, T, H, D).transpose(1, 2)
        dq, dk, dv = torch.autograd.grad(o, leaves, g)
        ctx.graph = None
        return torch.stack([t.transpose(1, 2) for t in (dq, dk, dv)], dim=2)


def attention_qkv(qkv: torch.Tensor) -> torch.Tensor:
    """Causal attention of a [B, T, 3, H, D] fused projection -> [B, T, H*D]."""
    if qkv.is_cuda:
        return _AttnQKV.apply(qkv)
    B, T, _, H, D = qkv.shape
    return _sdpa(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]).reshape(B, T, H * D)


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Causal attention over [B, T, H, D] q and [B, T, Hkv, D] k/v (GQA when
    Hkv < H); returns [B, T, H, D]."""
    return _sdpa(q, k, v)


class _AttnGQA(torch.autograd.Function):
    """Causal GQA attention over a fused [B, T, H + 2*Hkv, D] projection."""

    @staticmethod
    def forward(ctx, qkv, H, Hkv):
        B, T, _, D = qkv.shape
        with torch.enable_grad():
            parts = (qkv[:, :, :H], qkv[:, :, H:H + Hkv], qkv[:, :, H + Hkv:])
            leaves = [t.detach().transpose(1, 2).requires_grad_() for t in parts]
            o = F.scaled_dot_product_attention(*leaves, is_causal=True, enable_gqa=Hkv != H)
        ctx.graph = (leaves, o)
        ctx.shape = (B, T, H, D)
        return o.detach().transpose(1, 2).reshape(B, T, H * D)

    @staticmethod
    def backward(ctx, dout):
        leaves, o = ctx.graph
        B, T, H, D = ctx.shape
        g = dout.reshape(B, T, H, D).transpose(1, 2)
        dq, dk, dv = torch.autograd.grad(o, leaves, g)
        ctx.graph = None
        return torch.cat([t.transpose(1, 2) for t in (dq, dk, dv)], dim=2), None, None


def attention_gqa(qkv: torch.Tensor, n_head: int, n_kv_head: int) -> torch.Tensor:
    """Causal attention of a fused [B, T, H + 2*Hkv, D] projection -> [B, T, H*D]."""
    if qkv.is_cuda:
        return _AttnGQA.apply(qkv, n_head, n_kv_head)
    B, T, _, D = qkv.shape
    H, Hkv = n_head, n_kv_head
    o = _sdpa(qkv[:, :, :H], qkv[:, :, H:H + Hkv], qkv[:, :, H + Hkv:])
    return o.reshape(B, T, H * D)
