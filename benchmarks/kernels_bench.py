"""Bandwidth of the memory-bound kernels on one GPU.

    python benchmarks/kernels_bench.py --kernel adamw|rs_stats|grad_stats|cross_entropy|norm_bwd|add_norm
                                       [--n 268435456] [--iters 3]
                                       [--hidden 768] [--dtype fp16|bf16]   (norm kernels)

``cross_entropy`` times the forward + backward pair and then the forward
that writes the gradient itself (the engine's path).  ``rs_stats`` runs the fused reduce-scatter + statistics kernel over a
one-rank peer table (this GPU's own heap), i.e. the kernel's load/compute
structure without NVLink traffic.  Each launch is timed with CUDA events
(the working set of the default size is larger than L2); the result line
gives its algorithmic bytes, the median time and the achieved bandwidth as
a fraction of the measured HBM copy bandwidth (``MEASURED_PEAKS.json``,
else 6650 GB/s).  With few iterations it is also the target of an ncu
capture of one kernel.
"""

import argparse
import json
import os
import statistics
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from minispeed_b200.ops import _ext, kernels  # noqa: E402
from minispeed_b200.ops import nn as ops  # noqa: E402


def _hbm_gbs() -> float:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def timed(fn, iters, nbytes, label):
    """Time ``iters`` launches one by one; print one JSON result line."""
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    times = []
    for _ in range(iters):
        ev[0].record()
        fn()
        ev[1].record()
        torch.cuda.synchronize()
        times.append(ev[0].elapsed_time(ev[1]))
    ms = statistics.median(times)
    gbs = nbytes / ms / 1e6
    print(json.dumps({"kernel": label, "bytes": int(nbytes), "iters": iters,
                      "ms_median": round(ms, 4), "ms_min": round(min(times), 4),
                      "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / _hbm_gbs(), 3)}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True)
    ap.add_argument("--n", type=int, default=1 << 28)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--hidden", type=int, default=768, help="row width of the norm kernels")
    ap.add_argument("--dtype", choices=["fp16", "bf16"], default="fp16",
                    help="activation dtype of the norm kernels")
    a = ap.parse_args()
    C = _ext.get()
    dev = torch.device("cuda")
    n = a.n
    if a.kernel == "adamw":
        p, m, v = (torch.randn(n, device=dev) for _ in range(3))
        v.abs_()
        g = torch.randn(n, device=dev).half()
        po = torch.empty(n, device=dev, dtype=torch.half)
        stats = torch.tensor([0, 1, 1, 1, 0, 0, 0, 0], dtype=torch.float32, device=dev)
        fn = lambda: kernels.adamw_step(p, m, v, g, lr=1e-4, beta1=0.9, beta2=0.95, eps=1e-8,
                                        wd=0.1, bc1=0.5, bc2=0.5, grad_mul=1.0, stats=stats,
                                        param_out=po)
        timed(fn, a.iters, n * (12 + 2 + 12 + 2), "adamw")
    elif a.kernel == "grad_stats":
        g = torch.randn(n, device=dev).half()
        st = kernels.StepStats(dev)

        def fn():
            st.reset()
            st.accumulate(g, 1.0)
            st.finalize(1.0)
        timed(fn, a.iters, n * 2, "grad_stats")
    elif a.kernel == "rs_stats":
        heap = C.peer_alloc(n * 2 + 4096)
        try:
            heaps = torch.tensor([heap], dtype=torch.int64, device=dev)
            grad = C.tensor_from_ptr(heap, n, 1, dev.index or 0)
            grad.normal_()
            out = torch.empty(n, dtype=torch.float32, device=dev)
            st = kernels.StepStats(dev)

            def fn():
                st.reset()
                C.rs_stats(heaps, 0, 1, 0, out, 1, 1.0, None, -1, st.partials, st.flags, 0, 1184, True, 256)
            timed(fn, a.iters, n * (2 + 4), "rs_stats")
        finally:
            torch.cuda.synchronize()
            C.peer_free(heap)
    elif a.kernel == "cross_entropy":
        M, V = n // 65536 or 1, 50257
        logits = torch.randn(M, 50304, device=dev).half()[:, :V]
        tgt = torch.randint(0, V, (M,), device=dev)

        def fn():
            lg = logits.detach().requires_grad_()
            loss = ops.cross_entropy(lg, tgt)
            loss.backward()
        timed(fn, a.iters, M * V * 2 * 3, "cross_entropy fwd+bwd")
        # the engine's path: gradient written by the forward for the seed,
        # logits read once and written once
        seed = torch.ones(1, device=dev)

        def fused():
            lg = logits.detach().requires_grad_()
            with ops.expected_loss_grad(seed):
                loss = ops.cross_entropy(lg, tgt)
            loss.backward()
        timed(fused, a.iters, M * V * 2 * 2, "cross_entropy fwd+grad (one kernel)")
    elif a.kernel in ("norm_bwd", "add_norm"):
        Cd = a.hidden
        M = n // Cd
        dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
        x = torch.randn(M, Cd, device=dev).to(dt).requires_grad_()
        d = torch.randn(M, Cd, device=dev).to(dt).requires_grad_()
        w = torch.ones(Cd, device=dev).to(dt).requires_grad_()
        b = torch.zeros(Cd, device=dev).to(dt).requires_grad_()
        if a.kernel == "add_norm":
            fn = lambda: ops.add_norm(x.detach(), d.detach(), w, b)
            timed(fn, a.iters, M * Cd * 2 * 4, f"add_norm fwd {M}x{Cd} {a.dtype}")
        else:
            s, y = ops.add_norm(x, d, w, b)
            gy, gs = torch.randn_like(y), torch.randn_like(s)
            fn = lambda: torch.autograd.grad((s, y), (x,), (gs, gy), retain_graph=True)
            timed(fn, a.iters, M * Cd * 2 * 6, f"norm bwd {M}x{Cd} {a.dtype}")
    else:
        raise SystemExit(f"unknown kernel {a.kernel}")


if __name__ == "__main__":
    main()
