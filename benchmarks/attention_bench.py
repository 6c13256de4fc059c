"""Causal attention: native tcgen05 kernels vs PyTorch SDPA (cuDNN on B200).

    python benchmarks/attention_bench.py [--b 16 --t 1024 --h 12 --hkv 12 --d 64] [--iters 20]

Times forward and forward+backward of one layer's attention over a fused
qkv projection with CUDA events after warm-up; prints one JSON line per
implementation with the achieved TFLOP/s (causal FLOPs: 2*B*H*T^2*D forward,
2.5x that backward).
"""

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from minispeed_b200.ops import attention as A  # noqa: E402


def timeit(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--b", type=int, default=16)
    ap.add_argument("--t", type=int, default=1024)
    ap.add_argument("--h", type=int, default=12)
    ap.add_argument("--hkv", type=int, default=0)
    ap.add_argument("--d", type=int, default=64)
    ap.add_argument("--dtype", default="fp16")
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    hkv = a.hkv or a.h
    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    qkv = torch.randn(a.b, a.t, a.h + 2 * hkv, a.d, device="cuda").to(dt).requires_grad_()
    dout = torch.randn(a.b, a.t, a.h * a.d, device="cuda").to(dt)
    flops_f = 2.0 * a.b * a.h * a.t * a.t * a.d
    for impl in ("native", "sdpa"):
        os.environ["MSB_ATTN"] = impl
        fwd = lambda: A.attention_gqa(qkv.detach(), a.h, hkv)

        def fb():
            o = A.attention_gqa(qkv, a.h, hkv)
            torch.autograd.grad(o, (qkv,), dout)
        tf = timeit(fwd, a.iters)
        tfb = timeit(fb, a.iters)
        print(json.dumps({"impl": impl, "shape": [a.b, a.t, a.h, hkv, a.d], "dtype": a.dtype,
                          "fwd_ms": round(tf, 4), "fwd_tflops": round(flops_f / tf / 1e9, 1),
                          "fwd_bwd_ms": round(tfb, 4),
                          "bwd_ms": round(tfb - tf, 4),
                          "fwd_bwd_tflops": round(3.5 * flops_f / tfb / 1e9, 1)}), flush=True)


if __name__ == "__main__":
    main()
