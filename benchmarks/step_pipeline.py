"""Optimizer-step pipeline microbenchmark (one flat parameter group).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/step_pipeline.py \
        [--impl ours|reference] [--sizes 20,24,27,29,31] [--steps 30] [--dtype fp16]

Each step hands the engine a model-dtype gradient of 2**k elements (values
~N(0, 1e-3) times the 2**16 loss scale, pre-generated) and times ONLY
``engine.step()``: unscale, inf/nan check, reduction, global norm + clip,
AdamW on the ZeRO-2 shard and the parameter all-gather.  Rank 0 injects an
inf into its gradient on 1% of steps (those steps must be skipped by every
rank).  Device time with CUDA events, max over ranks.

Roofline of the fused path per rank: the slower of
  NVLink   2 * (W-1)/W * N * 2 bytes (16-bit gradient in, 16-bit params out)
           over the measured 770 GB/s per direction, and
  HBM      N*2 (local gradient reads) + (N/W)*(4*3*2 + 4) (AdamW state
           read+write, fp32 shard written) + N*2*... params written
           over the measured HBM bandwidth (MEASURED_PEAKS.json).
Prints one JSON line per size on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.nn as nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVLINK_GBS = 770.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:
        return 6650.0


class Flat(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.w = nn.Parameter(torch.zeros(n))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sizes", default="20,24,27,29,31")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16"])
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MINISPEED_DEVICE", f"cuda:{local}")
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        import minispeed as lib
    else:
        sys.path.insert(0, ROOT)
        import minispeed_b200 as lib
    lib.comm.init_distributed()
    dt = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    hbm = peaks()
    for k in (int(s) for s in args.sizes.split(",")):
        n = 1 << k
        model = Flat(n)
        cfg = {"train_micro_batch_size_per_gpu": 1, "gradient_clipping": 1.0,
               "dtype": args.dtype, "zero_optimization": {"stage": 2},
               "optimizer": {"type": "AdamW", "params": {"lr": 1e-4, "weight_decay": 0.01}},
               "steps_per_print": 10 ** 9}
        if args.dtype == "fp16":
            cfg["fp16"] = {"enabled": True, "initial_scale_power": 16, "loss_scale_window": 10 ** 6}
        engine = lib.initialize(model=model, config=cfg)
        gen = torch.Generator(device=dev).manual_seed(rank + 17)
        scale = 2.0 ** 16 if args.dtype == "fp16" else 1.0
        grad_src = (torch.randn(n, device=dev, generator=gen) * 1e-3 * scale).to(dt)
        p = model.w
        ms, skipped = [], 0
        for i in range(args.warmup + args.steps):
            # the gradient a backward pass would have left in p.grad (ours:
            # bind p.grad to the gradient arena as a forward would)
            if hasattr(engine, "_open_window"):
                engine._open_window()
            if p.grad is None:
                p.grad = grad_src.clone()
            else:
                p.grad.copy_(grad_src)
            inject = rank == 0 and i >= args.warmup and (i - args.warmup) % 100 == 10
            if inject:
                p.grad.view(-1)[n // 2] = float("inf")
            engine.micro_steps += 1
            torch.cuda.synchronize()
            if world > 1:
                torch.distributed.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            applied = engine.step()
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ms.append(a.elapsed_time(b))
                skipped += 0 if applied else 1
        t = torch.tensor([sum(ms) / len(ms)], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        mean_ms = float(t.item())
        esz = 2
        nv_bytes = 2 * (world - 1) / world * n * esz if world > 1 else 0.0
        hbm_bytes = n * esz + (n / world) * (4 * 6 + 4) + n * esz
        roof_ms = max(nv_bytes / (NVLINK_GBS * 1e9), hbm_bytes / (hbm * 1e9)) * 1e3
        if rank == 0:
            print(json.dumps({"impl": args.impl, "elements": n, "log2": k, "world": world,
                              "dtype": args.dtype, "ms_per_step": round(mean_ms, 4),
                              "roofline_ms": round(roof_ms, 4),
                              "fraction_of_roofline": round(roof_ms / mean_ms, 3),
                              "skipped_steps": skipped,
                              "collectives": getattr(engine, "collectives", "reference")}),
                  flush=True)
        if hasattr(engine, "close"):
            engine.close()
        del engine, model, grad_src, p
        torch.cuda.empty_cache()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
