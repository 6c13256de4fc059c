"""Run one tcgen05 GEMM shape a few times (profiling target).

    python benchmarks/gemm_one.py --m 16384 --n 768 --k 3072 [--layout fwd|dgrad|wgrad] [--iters 3]
"""

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from minispeed_b200.ops import gemm  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=768)
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--layout", default="fwd", choices=["fwd", "dgrad", "wgrad"])
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    kmaj = {"fwd": (True, True), "dgrad": (True, False), "wgrad": (False, False)}[a.layout]
    A = torch.randn(a.m, a.k, device="cuda").half()
    B = (torch.randn(a.n, a.k, device="cuda") * 0.02).half()
    A = A if kmaj[0] else A.t().contiguous()
    B = B if kmaj[1] else B.t().contiguous()
    out = torch.empty(a.m, a.n, device="cuda", dtype=torch.half)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for i in range(a.iters):
        ev[0].record()
        gemm.gemm(A, B, a_kmajor=kmaj[0], b_kmajor=kmaj[1], out=out)
        ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1])
        print(f"iter {i}: {ms:.4f} ms  {2.0 * a.m * a.n * a.k / ms / 1e9:.1f} TFLOP/s")
    gemm.check()


if __name__ == "__main__":
    main()
