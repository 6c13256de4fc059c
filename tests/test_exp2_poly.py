"""The FMA-pipe exp2 (``exp2_poly`` in ``csrc/common.cuh``) that the
attention kernels can use for part of their exponentials (the forward at run
time with ``MSB_ATTN_POLY=1|2``, the backward at build time with
``-DMSB_EXP2_POLY=n``; both off by default, where measured slower), evaluated
step by step in float32:
range reduction through the 1.5 * 2^23 rounding constant, degree-3 minimax
polynomial, exponent-field add.  Checks the relative error bound the kernel
comment states and the clamp at -125."""

import numpy as np

C = np.float32([0.99992806, 0.69326085, 0.24261115, 0.05517222])
MAGIC = np.float32(12582912.0)


def exp2_poly(x):
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    t = (x + MAGIC).astype(np.float32)
    f = (x - (t - MAGIC)).astype(np.float32)
    q = (C[3] * f + C[2]).astype(np.float32)
    q = (q * f + C[1]).astype(np.float32)
    q = (q * f + C[0]).astype(np.float32)
    bits = q.view(np.int32) + (t.view(np.int32) << np.int32(23))
    return bits.astype(np.int32).view(np.float32)


def test_relative_error_below_fp16_half_ulp():
    x = np.linspace(-124.0, 0.0, 2_000_001, dtype=np.float32)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(exp2_poly(x).astype(np.float64) / ref - 1.0)
    assert rel.max() < 8e-5 < 2.0 ** -12


def test_clamped_inputs_stay_normal_and_tiny():
    y = exp2_poly(np.float32([-125.0, -300.0, -1e30]))
    assert np.all(y > 0) and np.all(y < 1e-37)
    assert np.all(np.isfinite(y))
