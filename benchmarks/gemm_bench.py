"""GEMM throughput of the tcgen05 kernel vs the library product on the
GPT-2-small training shapes (M = 16 x 1024 tokens).

    python benchmarks/gemm_bench.py [--tokens 16384] [--iters 20]
    python benchmarks/gemm_bench.py --shape 16384,768,3072 --layout fwd [--iters 3]

Times each product with CUDA events after warm-up; inputs are re-used, the
operand set of each shape is < L2 for the small products, so this measures
kernel throughput (compare with the cuBLAS column, same conditions).

``--shape M,N,K`` runs one product of one layout (``fwd``: both operands
K-major; ``dgrad``: B N-major; ``wgrad``: both M-major) ``--iters`` times
without warm-up, each launch timed on its own, and prints one result line:
the target of an ncu capture of the kernel.
"""

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from minispeed_b200.ops import _ext, gemm  # noqa: E402


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


def one_shape(shape: str, layout: str, iters: int, dt) -> None:
    """One product, launched ``iters`` times, each timed on its own."""
    M, N, K = (int(v) for v in shape.split(","))
    kmaj = {"fwd": (True, True), "dgrad": (True, False), "wgrad": (False, False)}[layout]
    A = torch.randn(M, K, device="cuda").to(dt)
    B = (torch.randn(N, K, device="cuda") * 0.02).to(dt)
    A = A if kmaj[0] else A.t().contiguous()
    B = B if kmaj[1] else B.t().contiguous()
    out = torch.empty(M, N, device="cuda", dtype=dt)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    times = []
    for _ in range(iters):
        ev[0].record()
        gemm.gemm(A, B, a_kmajor=kmaj[0], b_kmajor=kmaj[1], out=out)
        ev[1].record()
        torch.cuda.synchronize()
        times.append(ev[0].elapsed_time(ev[1]))
    gemm.check()
    best = min(times)
    print(json.dumps({"gemm": layout, "M_N_K": [M, N, K], "iters": iters,
                      "ms": [round(t, 4) for t in times],
                      "best_tflops": round(2.0 * M * N * K / best / 1e9, 1)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--embd", type=int, default=768)
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16"])
    ap.add_argument("--shape", default=None, help="M,N,K: one product only")
    ap.add_argument("--layout", default="fwd", choices=["fwd", "dgrad", "wgrad"])
    args = ap.parse_args()
    if args.shape:
        one_shape(args.shape, args.layout, args.iters,
                  torch.float16 if args.dtype == "fp16" else torch.bfloat16)
        return
    T, C, V = args.tokens, args.embd, 50257
    Vp = 50304
    dt = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    rows = []
    shapes = [("qkv", 3 * C, C), ("proj", C, C), ("fc", 4 * C, C), ("fc2", C, 4 * C), ("head", V, C)]
    for name, N, K in shapes:
        x = torch.randn(T, K, device="cuda").to(dt)
        w = (torch.randn(N, K, device="cuda") * 0.02).to(dt)
        if name == "head":
            dy = torch.randn(T, Vp, device="cuda").to(dt)[:, :V]
        else:
            dy = torch.randn(T, N, device="cuda").to(dt)
        for kind in ("fwd", "dgrad", "wgrad"):
            if kind == "fwd" and name == "head":
                # the model's logits buffer: rows padded to a multiple of 64
                lg = torch.empty(T, Vp, device="cuda", dtype=dt)[:, :V]
                ours = lambda: gemm.gemm(x, w, a_kmajor=True, b_kmajor=True, out=lg)
                lib = lambda: torch.mm(x, w.t())
            elif kind == "fwd":
                ours = lambda: gemm.gemm(x, w, a_kmajor=True, b_kmajor=True)
                lib = lambda: torch.mm(x, w.t())
            elif kind == "dgrad":
                ours = lambda: gemm.gemm(dy, w, a_kmajor=True, b_kmajor=False)
                lib = lambda: torch.mm(dy, w)
            else:
                ours = lambda: gemm.gemm(dy, x, a_kmajor=False, b_kmajor=False)
                lib = lambda: torch.mm(dy.t(), x)
            flops = 2.0 * T * N * K
            t_o = timeit(ours, args.iters)
            gemm.check()
            t_l = timeit(lib, args.iters)
            mnk = [T if kind != "wgrad" else N,
                   N if kind == "fwd" else K,
                   K if kind == "fwd" else (N if kind == "dgrad" else T)]
            amn, bmn = {"fwd": (0, 0), "dgrad": (0, 1), "wgrad": (1, 1)}[kind]
            plan = _ext.get().gemm_cached_plan(*mnk, amn, bmn, 1 if dt == torch.float16 else 2, 0)
            rows.append({"gemm": f"{name}.{kind}", "M_N_K": mnk, "plan_bn_splits": list(plan),
                         "ours_ms": round(t_o, 4), "ours_tflops": round(flops / t_o / 1e9, 1),
                         "cublas_ms": round(t_l, 4), "cublas_tflops": round(flops / t_l / 1e9, 1)})
            print(json.dumps(rows[-1]), flush=True)
    tot_o = sum(r["ours_ms"] for r in rows)
    tot_l = sum(r["cublas_ms"] for r in rows)
    print(json.dumps({"total_ours_ms": round(tot_o, 3), "total_cublas_ms": round(tot_l, 3)}))


if __name__ == "__main__":
    main()
