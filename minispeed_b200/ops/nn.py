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

Reference: the layers of the example model (``examples/train_lm.py:62-115``:
``nn.Linear`` projections, ``nn.LayerNorm`` at ``:84``, ``:86`` and ``:105``,
``nn.GELU`` MLP at ``:88``, token + position embeddings) and its loss
(``F.cross_entropy`` at ``:246``).  ``swiglu``, RMSNorm and ``rope_`` serve the
Llama family, which the reference has no model for.
"""

from __future__ import annotations

import math
from contextlib import contextmanager
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import _ext, gemm

_COLSUM_CHUNKS = 256   # row chunks of a column-sum reduction
_NORM_BLOCKS = 296     # row chunks (blocks) of the norm-backward dw/db column sums


def _C():
    return _ext.get()


def _tc(x: torch.Tensor) -> bool:
    """GEMM-bearing ops run the tcgen05 kernels for 16-bit CUDA tensors; fp32
    models (a debugging configuration of the reference's GPU tests) run
    PyTorch's fp32 GEMM, since tcgen05 ``kind::f16`` takes 16-bit operands."""
    return x.is_cuda and x.dtype in (torch.float16, torch.bfloat16)


def _scratch(device, n: int) -> torch.Tensor:
    return torch.empty(n, dtype=torch.float32, device=device)


def as_matrix(t: torch.Tensor, n: int) -> torch.Tensor:
    """``t`` viewed as a row-major [rows, n] matrix with unit column stride;
    copies only when no such view exists (a padded leading dimension is kept)."""
    m = t.reshape(-1, n)
    if m.stride(-1) != 1 or (m.shape[0] > 1 and m.stride(0) < n):
        m = m.contiguous()
    return m


def grad_sink(p: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """The parameter's existing ``.grad`` if gradients can be accumulated into
    it in place (the engine binds every ``p.grad`` to a view of its flat
    gradient arena), else None.

    Backward kernels write into a sink directly (GEMM epilogue accumulate,
    column-sum accumulate) and report no gradient to autograd for that input,
    which is what autograd's own accumulation would have produced."""
    if p is None or not isinstance(p, torch.nn.Parameter):
        return None
    g = p.grad
    if g is None or g.dtype != p.dtype or g.shape != p.shape or not g.is_contiguous():
        return None
    return g


class _FinishQueue:
    """Column-sum finishes into gradient sinks, batched.

    A bias or norm-weight gradient is the column sum of fp32 partial rows
    that its backward kernel leaves; the finish that adds them into the
    gradient is a launch of its own, tiny and latency-bound (a GPT-2 small
    step has 98 of them).  Inside :func:`batched_colsums` (the engine's
    backward) finishes into sinks are queued instead and run together by
    ``colsum_finish_many``: one launch per flush.  A flush happens when the
    context exits normally, before a gradient bucket is handed to the
    collectives (:func:`flush_colsums`), when ``_BATCH`` finishes are queued,
    and before a finish whose sink, stream or dtype conflicts with the queue
    (two finishes into one sink in one launch would race).  The queue keeps
    each partial buffer alive until its flush has been launched.

    Autograd runs CUDA backward functions on its own thread while the caller
    waits in ``backward()``; the queue is shared module state, touched by one
    thread at a time."""

    _BATCH = 48

    def __init__(self):
        self.depth = 0
        self.clear()

    def clear(self):
        self.parts, self.nparts, self.outs = [], [], []
        self.sinks = set()
        self.stream = None

    def add(self, part: torch.Tensor, nparts: int, sink: torch.Tensor) -> None:
        st = torch.cuda.current_stream(sink.device)
        key = sink.data_ptr()
        if self.outs and (key in self.sinks or st != self.stream
                          or sink.dtype != self.outs[0].dtype):
            self.flush()
        if not self.outs:
            self.stream = st
        self.parts.append(part)
        self.nparts.append(int(nparts))
        self.outs.append(sink)
        self.sinks.add(key)
        if len(self.outs) >= self._BATCH:
            self.flush()

    def flush(self) -> None:
        if not self.outs:
            return
        with torch.cuda.stream(self.stream):
            _C().colsum_finish_many(self.parts, self.nparts, self.outs,
                                    [True] * len(self.outs))
        self.clear()


_finishes = _FinishQueue()


@contextmanager
def batched_colsums():
    """Queue column-sum finishes into gradient sinks while the block runs
    (a backward pass) and launch them batched; nests."""
    _finishes.depth += 1
    ok = False
    try:
        yield
        ok = True
    finally:
        _finishes.depth -= 1
        if _finishes.depth == 0:
            if ok:
                _finishes.flush()
            else:
                _finishes.clear()


def flush_colsums() -> None:
    """Launch the queued finishes now (the gradients they complete are about
    to be read)."""
    _finishes.flush()


def _finish_into(part: torch.Tensor, nparts: int, sink: torch.Tensor) -> None:
    """sink += the column sums of ``part``'s first ``nparts`` rows."""
    if _finishes.depth > 0:
        _finishes.add(part, nparts, sink)
    else:
        _C().colsum_finish(part, nparts, sink, True)


def _colsum(a2d: torch.Tensor, dtype, sink: Optional[torch.Tensor] = None
            ) -> Optional[torch.Tensor]:
    """Column sums of a [M, N] CUDA matrix (bias gradients); accumulated into
    ``sink`` (returns None) or returned as a new tensor."""
    n = a2d.shape[-1]
    part = _scratch(a2d.device, _COLSUM_CHUNKS * n)
    nb = _C().colsum_partial(a2d, part, _COLSUM_CHUNKS)
    if sink is not None:
        _finish_into(part, nb, sink)
        return None
    out = torch.empty(n, dtype=dtype, device=a2d.device)
    _C().colsum_finish(part, nb, out, False)
    return out


def _wgrad(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor) -> Optional[torch.Tensor]:
    """dW = dy^T x, accumulated into w's gradient sink when it has one."""
    sink = grad_sink(w)
    if sink is not None:
        gemm.linear_wgrad(dy2, x2, out=sink.view(sink.shape[0], -1), accumulate=True)
        return None
    return gemm.linear_wgrad(dy2, x2)


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
        ctx.params = (w, b)
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
        w_p, b_p = ctx.params
        dw = db = None
        sink = grad_sink(w_p)
        if sink is not None:
            _finish_into(dw_part, nb, sink)
        else:
            dw = torch.empty_like(w)
            _C().colsum_finish(dw_part, nb, dw, False)
        if ctx.has_bias:
            sink = grad_sink(b_p)
            if sink is not None:
                _finish_into(db_part, nb, sink)
            else:
                db = torch.empty_like(w)
                _C().colsum_finish(db_part, nb, db, False)
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
    def forward(ctx, x, w, b, pad):
        shp = x.shape
        x2 = as_matrix(x, shp[-1])
        N = w.shape[0]
        out = None
        if pad:
            # leading dimension rounded up to a multiple of `pad` elements so
            # that every row starts 16-byte aligned (TMA / vector access)
            ld = -(-N // pad) * pad
            out = torch.empty(x2.shape[0], ld, dtype=x.dtype, device=x.device)[:, :N]
        out = gemm.linear_fwd(x2, w, b, out=out)
        ctx.save_for_backward(x2, w)
        ctx.params = (w, b)
        ctx.shape = shp
        return out.view(*shp[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        w_p, b_p = ctx.params
        dy2 = as_matrix(dy, w.shape[0])
        dx = gemm.linear_dgrad(dy2, w) if ctx.needs_input_grad[0] else None
        dw = _wgrad(dy2, x2, w_p)
        db = _colsum(dy2, w.dtype, grad_sink(b_p)) if b_p is not None else None
        if dx is not None:
            dx = dx.view(ctx.shape)
        return dx, dw, db, None


class _MlpGelu(torch.autograd.Function):
    """fc2(gelu(fc(x))) with both GELU passes fused into GEMM epilogues:
    forward  fc : u = x W1^T + b1 and a = gelu(u) written by one epilogue
    backward fc2-dgrad: du = (dout W2) * gelu'(u) written by one epilogue."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2):
        shp = x.shape
        x2 = as_matrix(x, shp[-1])
        M, F_ = x2.shape[0], w1.shape[0]
        u = torch.empty(M, F_, dtype=x.dtype, device=x.device)
        a = torch.empty_like(u)
        gemm.gemm(x2, w1, a_kmajor=True, b_kmajor=True, bias=b1, out=u,
                  mode=gemm.EPI_BIAS_GELU, aux=a)
        out = gemm.linear_fwd(a, w2, b2)
        ctx.save_for_backward(x2, w1, u, a, w2)
        ctx.params = (w1, b1, w2, b2)
        ctx.shape = shp
        return out.view(*shp[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, dout):
        x2, w1, u, a, w2 = ctx.saved_tensors
        w1_p, b1_p, w2_p, b2_p = ctx.params
        d2 = as_matrix(dout, w2.shape[0])
        dw2 = _wgrad(d2, a, w2_p)
        db2 = _colsum(d2, w2.dtype, grad_sink(b2_p)) if b2_p is not None else None
        du = torch.empty_like(u)
        M, F_ = du.shape
        # the dGELU epilogue also leaves the column sums of du (fc bias
        # gradient), one partial row per 32 rows: no second read of du
        part = _scratch(du.device, -(-M // 32) * F_) if b1_p is not None else None
        gemm.gemm(d2, w2, a_kmajor=True, b_kmajor=False, out=du, mode=gemm.EPI_DGELU, aux=u,
                  colsum=part)
        dw1 = _wgrad(du, x2, w1_p)
        db1 = None
        if b1_p is not None:
            sink = grad_sink(b1_p)
            if sink is not None:
                _finish_into(part, -(-M // 32), sink)
            else:
                db1 = torch.empty(F_, dtype=w1.dtype, device=du.device)
                _C().colsum_finish(part, -(-M // 32), db1, False)
        dx = gemm.linear_dgrad(du, w1).view(ctx.shape) if ctx.needs_input_grad[0] else None
        return dx, dw1, db1, dw2, db2


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None,
           pad_out: int = 0) -> torch.Tensor:
    """``x @ w.T + b``.  ``pad_out`` > 0 allocates the output with its row
    stride rounded up to a multiple of ``pad_out`` (the returned tensor is a
    view with the logical width)."""
    if _tc(x):
        return _Linear.apply(x, w, b, pad_out)
    return F.linear(x, w, b)


def mlp_gelu(x: torch.Tensor, w1: torch.Tensor, b1: Optional[torch.Tensor], w2: torch.Tensor,
             b2: Optional[torch.Tensor]) -> torch.Tensor:
    """``fc2(gelu(fc(x)))`` (exact erf GELU)."""
    if _tc(x):
        return _MlpGelu.apply(x, w1, b1, w2, b2)
    return F.linear(F.gelu(F.linear(x, w1, b1)), w2, b2)


def linear_gelu(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
    """``gelu(x @ w.T + b)`` (pre-activation kept for backward)."""
    if _tc(x):
        return _LinearGelu.apply(x, w, b)
    return F.gelu(F.linear(x, w, b))


class _LinearGelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b):
        shp = x.shape
        x2 = as_matrix(x, shp[-1])
        u = torch.empty(x2.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        h = torch.empty_like(u)
        gemm.gemm(x2, w, a_kmajor=True, b_kmajor=True, bias=b, out=u,
                  mode=gemm.EPI_BIAS_GELU, aux=h)
        ctx.save_for_backward(x2, w, u)
        ctx.params = (w, b)
        ctx.shape = shp
        return h.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dh):
        x2, w, u = ctx.saved_tensors
        w_p, b_p = ctx.params
        du = torch.empty_like(u)
        _C().gelu_bwd(as_matrix(dh, w.shape[0]).contiguous(), u, du)
        dw = _wgrad(du, x2, w_p)
        db = _colsum(du, w.dtype, grad_sink(b_p)) if b_p is not None else None
        dx = gemm.linear_dgrad(du, w).view(ctx.shape) if ctx.needs_input_grad[0] else None
        return dx, dw, db


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
_LOSS_GRAD_HINT: list = [None]


@contextmanager
def expected_loss_grad(seed: Optional[torch.Tensor]):
    """Within this context, :func:`cross_entropy` on CUDA computes its
    gradient during the forward, for the upstream gradient ``seed`` (an fp32
    CUDA scalar: the backward seed the engine will use, i.e. loss scale /
    gradient-accumulation steps).  The backward then only checks the real
    upstream gradient against ``seed`` and rescales when they differ.  The
    logits are read from DRAM once instead of twice.  ``None`` turns it off."""
    prev = _LOSS_GRAD_HINT[0]
    _LOSS_GRAD_HINT[0] = seed
    try:
        yield
    finally:
        _LOSS_GRAD_HINT[0] = prev


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index, hint):
        V = logits.shape[-1]
        l2 = as_matrix(logits, V)
        M = l2.shape[0]
        t = targets.reshape(-1).contiguous()
        lse = torch.empty(M, dtype=torch.float32, device=logits.device)
        rows = torch.empty(M, dtype=torch.float32, device=logits.device)
        loss = torch.empty((), dtype=torch.float32, device=logits.device)
        inv = torch.empty(1, dtype=torch.float32, device=logits.device)
        if hint is not None:
            # the logits buffer becomes the gradient for upstream gradient `hint`
            _C().cross_entropy_fwd_grad(l2, t, lse, rows, loss, inv, hint, ignore_index)
        else:
            _C().cross_entropy_fwd(l2, t, lse, rows, loss, inv, ignore_index)
        ctx.save_for_backward(l2, t, lse, inv)
        ctx.hint = hint
        ctx.ignore_index = ignore_index
        ctx.shape = logits.shape
        return loss

    @staticmethod
    def backward(ctx, g):
        l2, t, lse, inv = ctx.saved_tensors
        go = g.float().reshape(1).contiguous()
        if ctx.hint is not None:
            _C().cross_entropy_grad_rescale(l2, go, ctx.hint)
        else:
            # the logits buffer is consumed in place: it becomes dlogits
            _C().cross_entropy_bwd(l2, t, lse, go, inv, ctx.ignore_index)
        ctx.hint = None
        return l2.view(ctx.shape), None, None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100
                  ) -> torch.Tensor:
    """Mean softmax cross-entropy in fp32 math over model-dtype logits.

    On CUDA the logits tensor is overwritten by its gradient (during backward,
    or during the forward inside :func:`expected_loss_grad`): it must not be
    used after the loss is computed."""
    if logits.is_cuda:
        hint = _LOSS_GRAD_HINT[0]
        if hint is not None and not (torch.is_grad_enabled() and logits.requires_grad
                                     and hint.device == logits.device):
            hint = None
        return _CrossEntropy.apply(logits, targets, ignore_index, hint)
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
        ctx.params = (wte, wpe)
        ctx.shapes = (wte.shape, None if wpe is None else wpe.shape, wte.dtype, T)
        return out

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        wte_shape, wpe_shape, dtype, T = ctx.shapes
        wte_p, wpe_p = ctx.params
        acc, touched = _embedding_accumulator(dout.device, wte_shape)
        # straight into the gradient arena when the parameter has a sink
        # (tied with the LM head: added to the head GEMM's wgrad), else into
        # a fresh zero gradient
        sink_te = grad_sink(wte_p)
        sink_pe = grad_sink(wpe_p) if wpe_shape is not None else None
        dwte = sink_te if sink_te is not None else torch.zeros(wte_shape, dtype=dtype,
                                                               device=dout.device)
        dwpe = None
        if wpe_shape is not None:
            dwpe = sink_pe if sink_pe is not None else torch.zeros(wpe_shape, dtype=dtype,
                                                                   device=dout.device)
        _C().embedding_bwd(dout.contiguous(), idx, acc, touched, dwte, True, dwpe, True, T)
        return (None, None if sink_te is not None else dwte,
                None if sink_pe is not None or dwpe is None else dwpe)


_EMB_ACC = {}


def _embedding_accumulator(device, shape) -> Tuple[torch.Tensor, torch.Tensor]:
    """The persistent fp32 scatter accumulator [V, C] and touched-row flags
    [V] of a device, zero between uses (the backward kernel clears the rows
    it reads).  Created on the first (eager) backward, before any CUDA-graph
    capture of the step."""
    key = (device, tuple(shape))
    buf = _EMB_ACC.get(key)
    if buf is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("embedding backward: run one eager step before capturing")
        buf = _EMB_ACC[key] = (torch.zeros(shape, dtype=torch.float32, device=device),
                               torch.zeros(shape[0], dtype=torch.uint8, device=device))
    return buf


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


class _RopeQK(torch.autograd.Function):
    """Rotary embedding of the q and k heads of a fused [B, T, H+2Hkv, D]
    projection (v passes through)."""

    @staticmethod
    def forward(ctx, qkv, cos, sin, H, Hkv):
        B, T, Ht, D = qkv.shape
        y = qkv.contiguous().clone()
        _C().rope(y, cos, sin, B * T, T, H + Hkv, D, Ht * D, False)
        ctx.save_for_backward(cos, sin)
        ctx.heads = (H, Hkv)
        return y

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        H, Hkv = ctx.heads
        B, T, Ht, D = dy.shape
        dx = dy.contiguous().clone()
        _C().rope(dx, cos, sin, B * T, T, H + Hkv, D, Ht * D, True)
        return dx, None, None, None, None


def rope_qk(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_head: int,
            n_kv_head: int) -> torch.Tensor:
    """Rotate the first ``n_head + n_kv_head`` heads (q and k) of a fused
    [B, T, H+2Hkv, D] projection."""
    if qkv.is_cuda:
        return _RopeQK.apply(qkv, cos, sin, n_head, n_kv_head)
    n = n_head + n_kv_head
    return torch.cat([rope(qkv[:, :, :n], cos, sin), qkv[:, :, n:]], dim=2)


def attention_gqa(qkv: torch.Tensor, n_head: int, n_kv_head: int) -> torch.Tensor:
    """Causal GQA attention of a fused [B, T, H+2Hkv, D] projection -> [B, T, H*D]."""
    from . import attention

    return attention.attention_gqa(qkv, n_head, n_kv_head)


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


def attention_qkv(qkv: torch.Tensor) -> torch.Tensor:
    """Causal attention of a fused [B, T, 3, H, D] projection -> [B, T, H*D]."""
    from . import attention

    return attention.attention_qkv(qkv)


def gelu_reference(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))


def gelu_grad_reference(u: torch.Tensor) -> torch.Tensor:
    cdf = 0.5 * (1.0 + torch.erf(u / math.sqrt(2.0)))
    return cdf + u * torch.exp(-0.5 * u * u) / math.sqrt(2.0 * math.pi)
