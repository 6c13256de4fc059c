"""GEMM entry points of the linear layers.

Three products per linear layer, all with 16-bit operands and fp32
accumulation:

* ``linear_fwd``   y[M,N]  = x[M,K] @ W[N,K]^T (+ b)   both operands K-major
* ``linear_dgrad`` dx[M,K] = dy[M,N] @ W[N,K]           W is N-major
* ``linear_wgrad`` dW[N,K] = dy[M,N]^T @ x[M,K]         both M-major

On CUDA they run the tcgen05/TMEM kernel of ``csrc/gemm_tcgen05.cu``
(TMA-fed shared-memory ring, accumulators in tensor memory, epilogue with
bias / accumulate; split-K or stream-K where the output has too few tiles
for whole waves, chosen per shape by timing the candidates once).  TMA needs 16-byte aligned
operand bases and row strides; an operand that is not (e.g. a parameter view
at an odd arena offset) is copied into an aligned buffer first.
``MSB_GEMM=torch`` selects the library product instead (comparison baseline
in the GEMM tests and benchmarks).

Reference: the ``nn.Linear`` layers of the example model
(``examples/train_lm.py:67-68``, ``:88``, ``:106``), whose products PyTorch
runs through cuBLAS there.

Each launch carries a device error word; kernels whose bounded waits time
out set it and return.  :func:`check` reads it (one host sync) and raises.
"""

from __future__ import annotations

import os
from typing import Dict, Optional

import torch

from . import _ext

_MODE = os.environ.get("MSB_GEMM", "auto")
TIMEOUT_S = float(os.environ.get("MSB_KERNEL_TIMEOUT_S", "2.0"))
_ERR: Dict[int, torch.Tensor] = {}


class KernelTimeoutError(RuntimeError):
    """A device-side bounded wait expired (the kernel returned early)."""


def error_word(device: torch.device) -> torch.Tensor:
    """The device status word that this device's GEMM and attention kernels set
    when a bounded wait gives up (allocated once per device)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = _ERR[idx] = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
    return t


def check(device: Optional[torch.device] = None) -> None:
    """Raise :class:`KernelTimeoutError` if any GEMM on ``device`` timed out."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    w = error_word(dev)
    code = int(w[0].item())
    if code:
        w.zero_()
        # an aborted stream-K launch can leave its tile counters raised
        _ext.get().gemm_reset_stream_k(w)
        raise KernelTimeoutError(f"tcgen05 gemm wait expired (code {code})")


def native_enabled() -> bool:
    """True unless ``MSB_GEMM=torch`` asked for the library product.

    With the native path selected, a missing or broken extension raises on
    the first CUDA GEMM (``_ext.get``) instead of falling back silently."""
    return _MODE != "torch"


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """Row-major view whose base and row stride are 16-byte aligned."""
    ok = (t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and (t.stride(0) * t.element_size()) % 16 == 0
          and t.stride(0) >= t.shape[1])
    if ok:
        return t
    rows, cols = t.shape
    ld = -(-cols // 8) * 8
    buf = torch.empty(rows, ld, dtype=t.dtype, device=t.device)[:, :cols]
    buf.copy_(t)
    return buf


EPI_PLAIN, EPI_BIAS_GELU, EPI_DGELU = 0, 1, 2


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_kmajor: bool, b_kmajor: bool,
         bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
         accumulate: bool = False, mode: int = EPI_PLAIN,
         aux: Optional[torch.Tensor] = None, plan: Optional[tuple] = None,
         colsum: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C[M,N] (+)= A @ B^T (+ bias) in the tcgen05 operand convention.

    ``a`` holds A as [M,K] (``a_kmajor``) or [K,M]; ``b`` holds B as [N,K]
    (``b_kmajor``) or [K,N].  Epilogue modes: ``EPI_BIAS_GELU`` stores
    u = A@B^T + bias into ``out`` and gelu(u) into ``aux``; ``EPI_DGELU``
    stores (A@B^T) * gelu'(aux) into ``out``.  ``plan=(bn, splits)`` replaces
    the tuned plan: bn 512 is the 2-CTA pair kernel (256 x 256 tiles), 256 or
    128 the 1-CTA kernel; splits 1-8 split K, -1 is stream-K (an even cut of
    all K slices over the resident pairs, pair kernel only).  ``colsum``
    (``EPI_DGELU`` only): an fp32 buffer of ceil(M/32) x N that receives the
    column sums of the stored output, one row per 32 output rows (finish
    with ``colsum_finish``): the bias gradient without re-reading C."""
    M = a.shape[0] if a_kmajor else a.shape[1]
    N = b.shape[0] if b_kmajor else b.shape[1]
    if out is None:
        out = torch.empty(M, N, dtype=a.dtype, device=a.device)
    if a.is_cuda and native_enabled():
        if a.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"tcgen05 gemm takes fp16 or bf16 operands, got {a.dtype}")
        bn, splits = plan if plan is not None else (0, 0)
        _ext.get().gemm(_tma_ready(a), _tma_ready(b), a_kmajor, b_kmajor, bias, out,
                        accumulate, error_word(a.device), TIMEOUT_S, mode, aux, bn, splits,
                        colsum)
        return out
    A = a if a_kmajor else a.t()
    B = b.t() if b_kmajor else b
    r = A.float() @ B.float()
    if bias is not None:
        r = r + bias.float()
    if mode == EPI_BIAS_GELU:
        u = r.to(out.dtype)
        out.copy_(u)
        aux.copy_(torch.nn.functional.gelu(u.float()).to(aux.dtype))
        return out
    if mode == EPI_DGELU:
        from .nn import gelu_grad_reference

        r = r.to(out.dtype).float() * gelu_grad_reference(aux.float())
        if colsum is not None:
            rows = r.to(out.dtype).float()
            pad = (-rows.shape[0]) % 32
            rows = torch.cat([rows, rows.new_zeros(pad, rows.shape[1])]) if pad else rows
            colsum.view(-1, N)[: rows.shape[0] // 32].copy_(rows.view(-1, 32, N).sum(1))
    if accumulate:
        out.copy_((out.float() + r).to(out.dtype))
    else:
        out.copy_(r.to(out.dtype))
    return out


def linear_fwd(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    return gemm(x, w, a_kmajor=True, b_kmajor=True, bias=bias, out=out)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return gemm(dy, w, a_kmajor=True, b_kmajor=False)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                 accumulate: bool = False) -> torch.Tensor:
    return gemm(dy, x, a_kmajor=False, b_kmajor=False, out=out, accumulate=accumulate)
