"""Causal self-attention (forward + backward) over a fused qkv projection.

``attention_qkv(qkv)`` takes the [B, T, 3, H, D] output of the fused qkv
projection (GPT-2) and ``attention_gqa(qkv, H, Hkv)`` the [B, T, H + 2*Hkv, D]
output of a grouped-query projection (Llama); both return [B, T, H*D], the
layout the output projection consumes.

On CUDA the forward and backward are this library's tcgen05 flash-attention
kernels (``csrc/attention_tcgen05.cu``): they read q, k and v straight out of
the projection output (no head-major copies), keep the scores in tensor
memory, skip the key tiles above the causal diagonal, and write the
gradient of the whole projection output (dq, dk, dv) in one buffer.  Head
dims 64 and 128 (GPT-2, Llama-3).  ``MSB_ATTN=sdpa`` selects PyTorch's SDPA
for every shape (comparison runs).

Reference: the example model's ``F.scaled_dot_product_attention(q, k, v,
is_causal=True)`` (``examples/train_lm.py:76``).
"""

from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from . import _ext, gemm


def native_enabled() -> bool:
    return os.environ.get("MSB_ATTN", "native").lower() != "sdpa"


def _sdpa(q, k, v):
    H, Hkv = q.shape[2], k.shape[2]
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
    if Hkv != H:
        rep = H // Hkv
        kt = kt.repeat_interleave(rep, dim=1)
        vt = vt.repeat_interleave(rep, dim=1)
    o = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True)
    return o.transpose(1, 2)


class _Flash(torch.autograd.Function):
    """Native causal attention over a fused [B, T, (H + 2*Hkv) * D] projection."""

    @staticmethod
    def forward(ctx, qkv, H, Hkv, D):
        B, T = qkv.shape[0], qkv.shape[1]
        W = (H + 2 * Hkv) * D
        q2 = qkv.reshape(B * T, W)
        if q2.stride(-1) != 1:
            q2 = q2.contiguous()
        out = torch.empty(B, T, H * D, dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty(B * H, T, dtype=torch.float32, device=qkv.device)
        scale = 1.0 / math.sqrt(D)
        _ext.get().attention_fwd(q2, 0, H * D, (H + Hkv) * D, out.view(B * T, H * D), lse, B, T,
                                 H, Hkv, D, scale, gemm.error_word(qkv.device), gemm.TIMEOUT_S)
        ctx.save_for_backward(q2, out, lse)
        ctx.dims = (B, T, H, Hkv, D, scale)
        ctx.qkv_shape = qkv.shape
        return out

    @staticmethod
    def backward(ctx, dout):
        q2, out, lse = ctx.saved_tensors
        B, T, H, Hkv, D, scale = ctx.dims
        d2 = dout.reshape(B * T, H * D)
        if d2.stride(-1) != 1 or d2.stride(0) % 8:
            d2 = d2.contiguous()
        dqkv = torch.empty_like(q2)
        delta = torch.empty(B * H, T, dtype=torch.float32, device=q2.device)
        dq_acc = torch.empty(B * T, H * D, dtype=torch.float32, device=q2.device)
        _ext.get().attention_bwd(q2, 0, H * D, (H + Hkv) * D, out.view(B * T, H * D), d2, lse,
                                 delta, dq_acc, dqkv, B, T, H, Hkv, D, scale,
                                 gemm.error_word(q2.device), gemm.TIMEOUT_S)
        return dqkv.view(ctx.qkv_shape), None, None, None


def _use_native(qkv: torch.Tensor, D: int) -> bool:
    return (qkv.is_cuda and native_enabled() and D in (64, 128)
            and qkv.dtype in (torch.float16, torch.bfloat16))


class _AttnQKV(torch.autograd.Function):
    """SDPA path over a [B, T, 3, H, D] projection (dq, dk, dv in one buffer)."""

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
    B, T, _, H, D = qkv.shape
    if _use_native(qkv, D):
        return _Flash.apply(qkv, H, H, D)
    if qkv.is_cuda:
        return _AttnQKV.apply(qkv)
    return _sdpa(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]).reshape(B, T, H * D)


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Causal attention over [B, T, H, D] q and [B, T, Hkv, D] k/v (GQA when
    Hkv < H); returns [B, T, H, D].  Separate tensors: the PyTorch path."""
    return _sdpa(q, k, v)


class _AttnGQA(torch.autograd.Function):
    """SDPA path over a fused [B, T, H + 2*Hkv, D] projection."""

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
    B, T, _, D = qkv.shape
    H, Hkv = n_head, n_kv_head
    if _use_native(qkv, D):
        return _Flash.apply(qkv, H, Hkv, D)
    if qkv.is_cuda:
        return _AttnGQA.apply(qkv, H, Hkv)
    o = _sdpa(qkv[:, :, :H], qkv[:, :, H:H + Hkv], qkv[:, :, H + Hkv:])
    return o.reshape(B, T, H * D)
