"""Autograd operators of the model zoo over the sm_100a kernels.

Every op has two definitions of the same math: the CUDA path (the kernels of
``minispeed_b200._C``) and a PyTorch path used for CPU tensors, which is
also the fp32 oracle of the GPU numerics tests.

Ops:
  ``add_norm``        fused residual add + LayerNorm/RMSNorm (returns the new
                      residual stream and the normalized activations)
  ``norm``            LayerNorm/RMSNorm without a residual
  ``linear``          x @ W^T + b through :mod:`.gemm`
  ``linear_gelu``     gelu(x @ W^T + b) (exact erf GELU, saves the pre-activation)
  ``swiglu``          silu(gate) * up on a fused [gate | up] projection
  ``cross_entropy``   fused softmax cross-entropy on model-dtype logits
  ``embedding``       token (+ learned position) embedding
  ``rope_``           rotary embedding on q/k views
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import _ext, gemm

_COLSUM_CHUNKS = 256   # row chunks of a column-sum reduction
_NORM_BLOCKS = 148 * 8  # norm backward blocks (one partial row of dw/db each)


def _C():
    return _ext.get()


def _scratch(device, n: int) -> torch.Tensor:
    return torch.empty(n, dtype=torch.float32, device=device)


def as_matrix(t: torch.Tensor, n: int) -> torch.Tensor:
    """``t`` viewed as a row-major [rows, n] matrix with unit column stride;
    copies only when no such view exists (a padded leading dimension is kept)."""
    m = t.reshape(-1, n)
    if m.stride(-1) != 1 or (m.shape[0] > 1 and m.stride(0) < n):
        m = m.contiguous()
    return m


def _colsum(a2d: torch.Tensor, dtype) -> torch.Tensor:
    """Column sums of a [M, N] CUDA matrix (bias gradients)."""
    n = a2d.shape[-1]
    part = _scratch(a2d.device, _COLSUM_CHUNKS * n)
    nb = _C().colsum_partial(a2d, part, _COLSUM_CHUNKS)
    out = torch.empty(n, dtype=dtype, device=a2d.device)
    _C().colsum_finish(part, nb, out)
    return out


# --------------------------------------------------------------- norms
class _AddNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, delta, w, b, eps, rms):
        C = x.shape[-1]
        M = x.numel() // C
        y = torch.empty_like(x)
        rstd = torch.empty(M, dtype=torch.float32, device=x.device)
        mean = None if rms else torch.empty(M, dtype=torch.float32, device=x.device)
        s = torch.empty_like(x) if delta is not None else None
        _C().add_norm_fwd(x, delta, w, b, s, y, mean, rstd, eps, rms)
        saved = s if s is not None else x
        ctx.save_for_backward(saved, w, mean, rstd)
        ctx.rms = rms
        ctx.has_delta = delta is not None
        ctx.has_bias = b is not None
        if s is not None:
            return s, y
        return y

    @staticmethod
    def backward(ctx, *grads):
        if ctx.has_delta:
            ds, dy = grads
        else:
            (dy,) = grads
            ds = None
        s, w, mean, rstd = ctx.saved_tensors
        C = s.shape[-1]
        dy = dy.contiguous()
        dx = torch.empty_like(s)
        dw_part = _scratch(s.device, _NORM_BLOCKS * C)
        db_part = None if ctx.rms else _scratch(s.device, _NORM_BLOCKS * C)
        if ds is not None:
            ds = ds.contiguous()
        nb = _C().norm_bwd(dy, s, w, mean, rstd, ds, dx, dw_part, db_part, ctx.rms,
                           _NORM_BLOCKS)
        dw = torch.empty_like(w)
        _C().colsum_finish(dw_part, nb, dw)
        db = None
        if ctx.has_bias:
            db = torch.empty_like(w)
            _C().colsum_finish(db_part, nb, db)
        if ctx.has_delta:
            return dx, dx, dw, db, None, None
        return dx, None, dw, db, None, None


def _norm_torch(x, w, b, eps, rms):
    xf = x.float()
    if rms:
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    else:
        y = F.layer_norm(xf, (x.shape[-1],), w.float(), None if b is None else b.float(), eps)
    return y.to(x.dtype)


def add_norm(x: torch.Tensor, delta: torch.Tensor, w, b, eps: float = 1e-5,
             rms: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """(s, y) with s = x + delta (residual stream) and y = norm(s)."""
    if x.is_cuda:
        return _AddNorm.apply(x.contiguous(), delta.contiguous(), w, b, eps, rms)
    s = x + delta
    return s, _norm_torch(s, w, b, eps, rms)


def norm(x: torch.Tensor, w, b, eps: float = 1e-5, rms: bool = False) -> torch.Tensor:
    if x.is_cuda:
        return _AddNorm.apply(x.contiguous(), None, w, b, eps, rms)
    return _norm_torch(x, w, b, eps, rms)


# -------------------------------------------------------------- linears
class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, act, pad):
        shp = x.shape
        x2 = as_matrix(x, shp[-1])
        N = w.shape[0]
        out = None
        if pad:
            # leading dimension rounded up to a multiple of `pad` elements so
            # that every row starts 16-byte aligned (TMA / vector access)
            ld = -(-N // pad) * pad
            out = torch.empty(x2.shape[0], ld, dtype=x.dtype, device=x.device)[:, :N]
        if act == "gelu":
            u = gemm.linear_fwd(x2, w, None)
            h = torch.empty_like(u)
            _C().bias_gelu_fwd(u, b, h)
            ctx.save_for_backward(x2, w, u)
            out = h
        else:
            out = gemm.linear_fwd(x2, w, b, out=out)
            ctx.save_for_backward(x2, w)
        ctx.act = act
        ctx.has_bias = b is not None
        ctx.shape = shp
        return out.view(*shp[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        if ctx.act == "gelu":
            x2, w, u = ctx.saved_tensors
        else:
            x2, w = ctx.saved_tensors
        dy2 = as_matrix(dy, w.shape[0])
        if ctx.act == "gelu":
            dy2 = dy2.contiguous()
            du = torch.empty_like(u)
            _C().gelu_bwd(dy2, u, du)
            dy2 = du
        dx = gemm.linear_dgrad(dy2, w) if ctx.needs_input_grad[0] else None
        dw = gemm.linear_wgrad(dy2, x2)
        db = _colsum(dy2, w.dtype) if ctx.has_bias else None
        if dx is not None:
            dx = dx.view(ctx.shape)
        return dx, dw, db, None, None


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None,
           pad_out: int = 0) -> torch.Tensor:
    """``x @ w.T + b``.  ``pad_out`` > 0 allocates the output with its row
    stride rounded up to a multiple of ``pad_out`` (the returned tensor is a
    view with the logical width)."""
    if x.is_cuda:
        return _Linear.apply(x, w, b, None, pad_out)
    return F.linear(x, w, b)


def linear_gelu(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
    if x.is_cuda:
        return _Linear.apply(x, w, b, "gelu", 0)
    return F.gelu(F.linear(x, w, b))


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        F_ = gu.shape[-1] // 2
        h = torch.empty(*gu.shape[:-1], F_, dtype=gu.dtype, device=gu.device)
        _C().swiglu_fwd(gu, h)
        ctx.save_for_backward(gu)
        return h

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        dgu = torch.empty_like(gu)
        _C().swiglu_bwd(dh.contiguous(), gu, dgu)
        return dgu


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gu[..., :F]) * gu[..., F:]`` for a fused gate/up projection."""
    if gu.is_cuda:
        return _SwiGLU.apply(gu.contiguous())
    g, u = gu.chunk(2, dim=-1)
    return (F.silu(g.float()) * u.float()).to(gu.dtype)


# -------------------------------------------------------- cross entropy
class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index):
        V = logits.shape[-1]
        l2 = as_matrix(logits, V)
        M = l2.shape[0]
        t = targets.reshape(-1).contiguous()
        lse = torch.empty(M, dtype=torch.float32, device=logits.device)
        rows = torch.empty(M, dtype=torch.float32, device=logits.device)
        loss = torch.empty((), dtype=torch.float32, device=logits.device)
        inv = torch.empty(1, dtype=torch.float32, device=logits.device)
        _C().cross_entropy_fwd(l2, t, lse, rows, loss, inv, ignore_index)
        ctx.save_for_backward(l2, t, lse, inv)
        ctx.ignore_index = ignore_index
        ctx.shape = logits.shape
        return loss

    @staticmethod
    def backward(ctx, g):
        l2, t, lse, inv = ctx.saved_tensors
        # the logits buffer is consumed in place: it becomes dlogits
        _C().cross_entropy_bwd(l2, t, lse, g.float().reshape(1).contiguous(), inv,
                               ctx.ignore_index)
        return l2.view(ctx.shape), None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100
                  ) -> torch.Tensor:
    """Mean softmax cross-entropy in fp32 math over model-dtype logits.

    On CUDA the logits tensor is overwritten by its gradient during backward
    (it must not be used after ``loss.backward()``)."""
    if logits.is_cuda:
        return _CrossEntropy.apply(logits, targets, ignore_index)
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1),
                           ignore_index=ignore_index)


# ------------------------------------------------------------ embedding
class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, wte, wpe):
        B, T = idx.shape
        C = wte.shape[1]
        out = torch.empty(B, T, C, dtype=wte.dtype, device=wte.device)
        idx = idx.contiguous()
        _C().embedding_fwd(idx, wte, wpe, out, T)
        ctx.save_for_backward(idx)
        ctx.shapes = (wte.shape, None if wpe is None else wpe.shape, wte.dtype, T)
        return out

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        wte_shape, wpe_shape, dtype, T = ctx.shapes
        dwte = torch.zeros(wte_shape, dtype=torch.float32, device=dout.device)
        dwpe = None if wpe_shape is None else torch.zeros(wpe_shape, dtype=torch.float32,
                                                          device=dout.device)
        _C().embedding_bwd(dout.contiguous(), idx, dwte, dwpe, T)
        return None, dwte.to(dtype), None if dwpe is None else dwpe.to(dtype)


def embedding(idx: torch.Tensor, wte: torch.Tensor, wpe: Optional[torch.Tensor] = None
              ) -> torch.Tensor:
    """``wte[idx] (+ wpe[:T])``."""
    if wte.is_cuda:
        return _Embedding.apply(idx, wte, wpe)
    x = F.embedding(idx, wte)
    if wpe is not None:
        x = x + wpe[: idx.shape[1]]
    return x


# ------------------------------------------------------------------ rope
def rope_tables(T: int, D: int, theta: float, device) -> Tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64, device=device) / D))
    ang = torch.arange(T, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cos(ang).float().contiguous(), torch.sin(ang).float().contiguous()


class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin):
        B, T, H, D = x.shape
        y = x.contiguous().clone()
        _C().rope(y, cos, sin, B * T, T, H, D, H * D, False)
        ctx.save_for_backward(cos, sin)
        return y

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        B, T, H, D = dy.shape
        dx = dy.contiguous().clone()
        _C().rope(dx, cos, sin, B * T, T, H, D, H * D, True)
        return dx, None, None


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding of ``x`` [B, T, H, D] (rotate-half convention)."""
    if x.is_cuda:
        return _Rope.apply(x, cos, sin)
    D = x.shape[-1]
    x1, x2 = x[..., : D // 2].float(), x[..., D // 2:].float()
    c = cos[: x.shape[1]][None, :, None, :]
    s = sin[: x.shape[1]][None, :, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


# ------------------------------------------------------------- attention
def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Causal attention over [B, T, H, D] q and [B, T, Hkv, D] k/v (GQA when
    Hkv < H); returns [B, T, H, D]."""
    from . import attention

    return attention.causal_attention(q, k, v)


def gelu_reference(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))
